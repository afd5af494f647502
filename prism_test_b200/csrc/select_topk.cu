// Exact per-row top-k over an fp32 score matrix, sorted like torch.topk
// (descending score; ties broken by ascending key index so results are
// deterministic).
//
// Reference semantics: scores.topk(k, dim=-1) in ReAttentionMethod._dense_topk
// (eval_harness/attention_methods/reattention.py:486-498) and the sorted 4-wide
// merge of the Triton kernel (eval_harness/kernels/bitonic_merge_wrapper.py:36-52),
// generalised here to any k <= 16384.
//
// Scores are compared through an order-preserving 32-bit key (NaN largest, as in
// torch.topk); a candidate is (key << 32) | ~index, so one unsigned 64-bit
// comparison orders by score and then by ascending index.
//
// Fast path: one thread-block cluster of 4 CTAs per row (select_topk_cluster_kernel
// below): an exact radix threshold from cluster-summed histograms, an append of
// the keys above it to a per-row candidate buffer, and a counting sort on the
// leader. General path (no candidate buffer, and the fallback when exact key ties
// alone exceed 16384 candidates): radix select with 12/12/8-bit digits on one
// block, compaction, shared-memory bitonic sort; massive ties at the k-th key are
// resolved in column order.
#include <cooperative_groups.h>

#include <cstddef>

#include "common.cuh"
#include "kernels.h"

namespace cg = cooperative_groups;

namespace prism {
namespace {

constexpr int kThreads = 1024;
constexpr int kCluster = 4;
constexpr int kBins = 4096;        // 12-bit radix digit histogram
constexpr int kFineBins = 8192;    // counting-sort bins of the fast path
constexpr int kCap = kSelectMaxK;  // 16384 sorted entries (128 KB)
// From this many rows on, one CTA per row (enough rows to fill the SMs) beats a
// 4-CTA cluster per row, whose grid would take several waves.
constexpr int64_t kRowKernelMinRows = 64;

struct SelectSmem {
  uint64_t buf[kCap];     // candidates (leader) / private level histograms / general path
  uint32_t hist[kFineBins];
  uint16_t perm[kCap];    // candidate numbers in fine-bin order (leader)
  uint32_t warp_tot[32];
  uint32_t bin, above, bcount;  // threshold digit (the leader's answer)
  uint32_t gt[4], acc[4];       // per cluster CTA: keys above the digit; above earlier digits
  uint32_t base[4], total;      // first candidate slot of each CTA; candidates of the row
  uint32_t kmax;          // largest key of the row
  uint32_t woff;          // candidate slots taken inside this CTA's range
  uint32_t thr, cbase;    // sampled threshold; this CTA's first slot (fast path)
  uint32_t count;         // candidates of the row (the leader's slot counter, fast path)
  uint32_t rlen[17], roff[17];  // run merge: prefix length and staging offset of each run
  unsigned long long rthr;      // run merge: threshold candidate
  uint32_t big;           // largest fine bin
  int ncand;
  uint32_t fcount[4], fkmax[4];  // fast path: every cluster CTA's candidates and largest key
  uint32_t nsamp;         // fast path: sampled columns of the row
};

__device__ __forceinline__ uint64_t pack_cand(uint32_t key, uint32_t idx) {
  return (uint64_t(key) << 32) | uint64_t(~idx);
}

// Visit every (key, index) of columns [c0, c1) of a row (c0 % 4 == 0).
template <typename F>
__device__ __forceinline__ void for_each_key(const SelectArgs& a, int64_t row, int64_t c0,
                                             int64_t c1, F&& f) {
  const float* sc = a.scores + row * a.ld;
  const int32_t* ix = a.idx_in ? a.idx_in + row * a.ld : nullptr;
  const int64_t e4_end = c1 >> 2;
  for (int64_t e4 = (c0 >> 2) + threadIdx.x; e4 < e4_end; e4 += kThreads) {
    const float4 v = reinterpret_cast<const float4*>(sc)[e4];
    const int64_t e = e4 << 2;
    if (ix) {
      const int4 iv = reinterpret_cast<const int4*>(ix)[e4];
      f(float_to_okey(v.x), uint32_t(iv.x));
      f(float_to_okey(v.y), uint32_t(iv.y));
      f(float_to_okey(v.z), uint32_t(iv.z));
      f(float_to_okey(v.w), uint32_t(iv.w));
    } else {
      f(float_to_okey(v.x), uint32_t(e));
      f(float_to_okey(v.y), uint32_t(e + 1));
      f(float_to_okey(v.z), uint32_t(e + 2));
      f(float_to_okey(v.w), uint32_t(e + 3));
    }
  }
  for (int64_t e = (e4_end << 2) + threadIdx.x; e < c1; e += kThreads)
    f(float_to_okey(sc[e]), ix ? uint32_t(ix[e]) : uint32_t(e));
}

// Block-wide exclusive scan of one value per thread.
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t v, SelectSmem& sm, uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sm.warp_tot[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = sm.warp_tot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    sm.warp_tot[lane] = w;
  }
  __syncthreads();
  const uint32_t warp_excl = warp ? sm.warp_tot[warp - 1] : 0u;
  if (total) *total = sm.warp_tot[31];
  const uint32_t r = warp_excl + x - v;
  __syncthreads();
  return r;
}

// Largest bin b with sum(hist[b..nbins)) >= need; sm.bin / sm.above (count above b).
// `hist` (default sm.hist): the histogram to search.
__device__ void find_bin(SelectSmem& sm, int nbins, uint32_t need, const uint32_t* hist = nullptr) {
  const uint32_t* hh = hist ? hist : sm.hist;
  const int t = threadIdx.x;
  const int hi_bin = nbins - 1 - 4 * t;
  uint32_t local = 0;
  if (hi_bin >= 0) {
#pragma unroll
    for (int u = 0; u < 4; ++u) local += (hi_bin - u >= 0) ? hh[hi_bin - u] : 0u;
  }
  if (t == 0) {
    sm.bin = 0;
    sm.above = 0;
  }
  const uint32_t excl = block_excl_scan(local, sm, nullptr);
  if (hi_bin >= 0 && excl < need && excl + local >= need) {
    uint32_t c = excl;
    for (int u = 0; u < 4; ++u) {
      const int bb = hi_bin - u;
      const uint32_t h = hh[bb];
      if (c + h >= need) {
        sm.bin = uint32_t(bb);
        sm.above = c;
        break;
      }
      c += h;
    }
  }
  __syncthreads();
}

__device__ __forceinline__ void zero_hist(SelectSmem& sm, int nbins) {
  for (int i = threadIdx.x; i < nbins; i += kThreads) sm.hist[i] = 0u;
  __syncthreads();
}

// Descending bitonic sort of sm.buf[0, n) (n <= kCap), padding with 0.
__device__ void block_bitonic_sort(SelectSmem& sm, int n) {
  int P = 1;
  while (P < n) P <<= 1;
  for (int i = n + threadIdx.x; i < P; i += kThreads) sm.buf[i] = 0ull;
  __syncthreads();
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < (P >> 1); i += kThreads) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool desc = (lo & size) == 0;
        const uint64_t x = sm.buf[lo], y = sm.buf[hi];
        if ((x < y) == desc) {
          sm.buf[lo] = y;
          sm.buf[hi] = x;
        }
      }
      __syncthreads();
    }
  }
}

__device__ void write_out(const SelectArgs& a, int64_t row, const SelectSmem& sm) {
  int32_t* oi = a.out_idx + row * a.k;
  float* os = a.out_scores ? a.out_scores + row * a.k : nullptr;
  const int64_t base = a.idx_in ? 0 : a.index_base;
  for (int t = threadIdx.x; t < a.k; t += kThreads) {
    const uint64_t u = sm.buf[t];
    oi[t] = int32_t(int64_t(~uint32_t(u)) + base);
    if (os) os[t] = okey_to_float(uint32_t(u >> 32));
  }
}

// General exact path for one row on one 1024-thread block (radix select on the
// full row, compaction into sm.buf, bitonic sort).
__device__ void select_row_general(const SelectArgs& a, int64_t row, SelectSmem& sm) {
  const uint32_t kk = uint32_t(a.k);
  zero_hist(sm, kBins);
  if (threadIdx.x == 0) sm.ncand = 0;
  for_each_key(a, row, 0, a.n, [&](uint32_t key, uint32_t) { atomicAdd(&sm.hist[key >> 20], 1u); });
  __syncthreads();
  find_bin(sm, kBins, kk);
  const uint32_t b1 = sm.bin, above1 = sm.above;
  const uint32_t total1 = above1 + sm.hist[b1];
  uint32_t thr;
  bool tie_pass = false;
  uint32_t tie_key = 0, need_ties = 0;
  if (total1 <= uint32_t(kCap)) {
    thr = b1 << 20;
  } else {
    __syncthreads();
    zero_hist(sm, kBins);
    for_each_key(a, row, 0, a.n, [&](uint32_t key, uint32_t) {
      if ((key >> 20) == b1) atomicAdd(&sm.hist[(key >> 8) & 0xfffu], 1u);
    });
    __syncthreads();
    find_bin(sm, kBins, kk - above1);
    const uint32_t b2 = sm.bin, above2 = sm.above;
    const uint32_t pre24 = (b1 << 12) | b2;
    if (above1 + above2 + sm.hist[b2] <= uint32_t(kCap)) {
      thr = pre24 << 8;
    } else {
      __syncthreads();
      zero_hist(sm, 256);
      for_each_key(a, row, 0, a.n, [&](uint32_t key, uint32_t) {
        if ((key >> 8) == pre24) atomicAdd(&sm.hist[key & 0xffu], 1u);
      });
      __syncthreads();
      find_bin(sm, 256, kk - above1 - above2);
      const uint32_t b3 = sm.bin, above3 = sm.above;
      const uint32_t T = (pre24 << 8) | b3;
      const uint32_t A = above1 + above2 + above3;
      if (A + sm.hist[b3] <= uint32_t(kCap)) {
        thr = T;
      } else {
        thr = T;  // keys > T (A < kk of them; none when T is NaN's key), then ties in column order
        tie_pass = true;
        tie_key = T;
        need_ties = kk - A;
      }
    }
  }
  __syncthreads();
  for_each_key(a, row, 0, a.n, [&](uint32_t key, uint32_t idx) {
    if (tie_pass ? key > tie_key : key >= thr) {
      const int slot = atomicAdd(&sm.ncand, 1);
      if (slot < kCap) sm.buf[slot] = pack_cand(key, idx);
    }
  });
  __syncthreads();
  if (tie_pass) {
    const int base0 = min(sm.ncand, kCap);
    uint32_t taken = 0;
    const float* sc = a.scores + row * a.ld;
    const int32_t* ix = a.idx_in ? a.idx_in + row * a.ld : nullptr;
    for (int64_t e0 = 0; e0 < a.n && taken < need_ties; e0 += kThreads) {
      const int64_t e = e0 + threadIdx.x;
      uint32_t key = 0, idx = 0;
      bool tie = false;
      if (e < a.n) {
        key = float_to_okey(sc[e]);
        idx = ix ? uint32_t(ix[e]) : uint32_t(e);
        tie = key == tie_key;
      }
      uint32_t chunk_total;
      const uint32_t rank = block_excl_scan(tie ? 1u : 0u, sm, &chunk_total);
      if (tie && taken + rank < need_ties && base0 + int(taken + rank) < kCap)
        sm.buf[base0 + taken + rank] = pack_cand(key, idx);
      taken += chunk_total;
    }
    __syncthreads();
    if (threadIdx.x == 0) sm.ncand = base0 + int(min(taken, need_ties));
    __syncthreads();
  }
  int nc = sm.ncand;
  if (nc > kCap) {
    if (threadIdx.x == 0) set_status(a.status, kStatusCapacity);
    nc = kCap;
  }
  block_bitonic_sort(sm, nc);
  write_out(a, row, sm);
}


// ---- cluster select ------------------------------------------------------------------
// Thread t of CTA r holds, for pass p, the kKeys keys of columns
//   p * kPass + r * kThreads * kKeys + ((j >> 2) * kThreads + t) * 4 + (j & 3),  j < kKeys
// (coalesced float4 loads). Key 0 marks a column beyond n: no fp32 value maps to 0.
constexpr int kKeys = 32;
constexpr int kPass = kCluster * kThreads * kKeys;  // 131072 columns per pass
constexpr int kLevelBins = 2048;                    // 11-bit digits (10 at the last level)
constexpr int kPriv = 8;                            // private histograms, one per lane & 7
constexpr int kPrivStride = kLevelBins + 4;         // copies start in different banks
constexpr int kRankMax = 256;                       // larger fine bins: bitonic sort instead

__device__ __forceinline__ void load_keys(const float* sc, int64_t base, int64_t n,
                                          uint32_t (&kv)[kKeys]) {
#pragma unroll
  for (int u = 0; u < kKeys / 4; ++u) {
    const int64_t e = base + (int64_t(u * kThreads + int(threadIdx.x)) << 2);
    if (e + 4 <= n) {
      const float4 v = *reinterpret_cast<const float4*>(sc + e);
      kv[4 * u + 0] = float_to_okey(v.x);
      kv[4 * u + 1] = float_to_okey(v.y);
      kv[4 * u + 2] = float_to_okey(v.z);
      kv[4 * u + 3] = float_to_okey(v.w);
    } else {
#pragma unroll
      for (int x = 0; x < 4; ++x) kv[4 * u + x] = e + x < n ? float_to_okey(sc[e + x]) : 0u;
    }
  }
}

// load_keys in two halves: the loads are issued first (raw fp32, absent columns
// as NaN placeholders) and converted later, so that other work can overlap them.
__device__ __forceinline__ void load_raw(const float* sc, int64_t base, int64_t n, float4 (&v)[kKeys / 4]) {
#pragma unroll
  for (int u = 0; u < kKeys / 4; ++u) {
    const int64_t e = base + (int64_t(u * kThreads + int(threadIdx.x)) << 2);
    if (e + 4 <= n) {
      v[u] = __ldcg(reinterpret_cast<const float4*>(sc + e));
    } else {
      v[u].x = e + 0 < n ? sc[e + 0] : 0.f;
      v[u].y = e + 1 < n ? sc[e + 1] : 0.f;
      v[u].z = e + 2 < n ? sc[e + 2] : 0.f;
      v[u].w = e + 3 < n ? sc[e + 3] : 0.f;
    }
  }
}
__device__ __forceinline__ void convert_raw(const float4 (&v)[kKeys / 4], int64_t base, int64_t n,
                                            uint32_t (&kv)[kKeys]) {
  if (base + int64_t(kThreads) * kKeys <= n) {  // every column of this CTA's pass exists
#pragma unroll
    for (int u = 0; u < kKeys / 4; ++u) {
      kv[4 * u + 0] = float_to_okey(v[u].x);
      kv[4 * u + 1] = float_to_okey(v[u].y);
      kv[4 * u + 2] = float_to_okey(v[u].z);
      kv[4 * u + 3] = float_to_okey(v[u].w);
    }
    return;
  }
#pragma unroll
  for (int u = 0; u < kKeys / 4; ++u) {
    const int64_t e = base + (int64_t(u * kThreads + int(threadIdx.x)) << 2);
    kv[4 * u + 0] = e + 0 < n ? float_to_okey(v[u].x) : 0u;
    kv[4 * u + 1] = e + 1 < n ? float_to_okey(v[u].y) : 0u;
    kv[4 * u + 2] = e + 2 < n ? float_to_okey(v[u].z) : 0u;
    kv[4 * u + 3] = e + 3 < n ? float_to_okey(v[u].w) : 0u;
  }
}

__device__ __forceinline__ int64_t key_column(int64_t base, int j) {
  return base + (int64_t((j >> 2) * kThreads + int(threadIdx.x)) << 2) + (j & 3);
}

// Split cluster barrier (arrive publishes this CTA's prior writes; wait acquires
// everyone's). Every thread of every CTA alternates arrive and wait.
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Leader, over the per-CTA histograms hist[r * kLevelBins + digit]: the largest
// digit b with (keys in digits >= b) >= need, the keys above it (sm.above) and in
// it (sm.bcount), and each CTA's count of keys in digits above b (sm.gt[r]).
__device__ void leader_find(SelectSmem& sm, int nb, uint32_t need) {
  const int t = threadIdx.x, lane = t & 31;
  uint32_t v[2] = {0u, 0u};
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int bb = nb - 1 - 2 * t - u;
    if (bb >= 0)
#pragma unroll
      for (int r = 0; r < kCluster; ++r) v[u] += sm.hist[r * kLevelBins + bb];
  }
  if (t == 0) {
    sm.bin = 0;
    sm.above = 0;
    sm.bcount = 0;
  }
  if (t < kCluster) sm.gt[t] = 0;
  const uint32_t excl = block_excl_scan(v[0] + v[1], sm, nullptr);
  if (excl < need && excl + v[0] + v[1] >= need) {
    const int bb = nb - 1 - 2 * t;
    const bool first = excl + v[0] >= need;
    sm.bin = uint32_t(first ? bb : bb - 1);
    sm.above = first ? excl : excl + v[0];
    sm.bcount = first ? v[0] : v[1];
  }
  __syncthreads();
  const int b = int(sm.bin);
#pragma unroll
  for (int r = 0; r < kCluster; ++r) {
    uint32_t c = 0;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int bb = nb - 1 - 2 * t - u;
      if (bb > b) c += sm.hist[r * kLevelBins + bb];
    }
    c = __reduce_add_sync(0xffffffffu, c);
    if (lane == 0 && c) atomicAdd(&sm.gt[r], c);
  }
  __syncthreads();
}

// Smallest fine bin f whose end (sm.hist after the scatter) exceeds position p.
__device__ __forceinline__ uint32_t bin_of_position(const SelectSmem& sm, uint32_t p) {
  uint32_t lo = 0, hi = kFineBins - 1;
  while (lo < hi) {
    const uint32_t mid = (lo + hi) >> 1;
    if (sm.hist[mid] > p) hi = mid;
    else lo = mid + 1;
  }
  return lo;
}

// ---- fast path: sampled threshold, candidates replicated in every CTA -------------------
constexpr int kSampleBins = 4096;                // 12-bit digits (key >> 20)
constexpr int kSampleCopies = 4;                 // private copies, one per lane & 3
constexpr int kSampleStride = kSampleBins + 4;
// Row sample of the fast paths: 8 consecutive columns of every 2^cshift (128 for a
// row held in registers, 256 for longer rows), at an offset hashed from the chunk
// number. Every CTA of a cluster reads the same columns and so computes the same
// threshold on its own, with no exchange: the lower edge of the 12-bit key digit
// holding sample rank 1.1 e + 4 sqrt(e) + 8, e = k * ns / n the expected sample
// rank of the k-th key (1 = every key when that rank exceeds the sample). Private
// histogram copies in sm.buf (zero on entry), the sum in sm.hist.
// `after_issue` runs once, after the first sample loads are issued (the caller's
// own loads then queue behind them).
// Visits every sampled key: f(order key). `after_issue` runs once, after the first
// loads are issued.
// With nparts > 1, only the chunks g with g % nparts == part.
template <typename F, typename G>
__device__ __forceinline__ void for_each_sample(const SelectArgs& a, const float* sc, int cshift,
                                                F&& f, G&& after_issue, int part = 0, int nparts = 1) {
  const int tid = threadIdx.x;
  const int oshift = 32 - (cshift - 3);  // hash -> one of chunk / 8 offsets
  const int64_t ngroups = (a.n + (int64_t(1) << cshift) - 1) >> cshift;
  const int64_t nmine = (ngroups - part + nparts - 1) / nparts;  // this part's chunks
  for (int64_t g0 = 0; g0 < nmine; g0 += int64_t(kThreads) * 2) {
    float4 v[2][2];
    int64_t e[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int64_t gi = g0 + int64_t(u) * kThreads + tid;
      const int64_t g = gi < nmine ? gi * nparts + part : ngroups;
      e[u] = (g << cshift) + 8 * int64_t((uint32_t(g) * 0x9E3779B1u) >> oshift);
      const bool full = g < ngroups && e[u] + 8 <= a.n;
      v[u][0] = full ? __ldcg(reinterpret_cast<const float4*>(sc + e[u])) : make_float4(0.f, 0.f, 0.f, 0.f);
      v[u][1] = full ? __ldcg(reinterpret_cast<const float4*>(sc + e[u] + 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
      if (!full) e[u] = g < ngroups ? -e[u] - 1 : INT64_MIN;  // partial or absent chunk
    }
    if (g0 == 0) after_issue();
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (e[u] == INT64_MIN) continue;
      const bool full = e[u] >= 0;
      const int64_t eb = full ? e[u] : -e[u] - 1;
      const float fv[8] = {v[u][0].x, v[u][0].y, v[u][0].z, v[u][0].w,
                           v[u][1].x, v[u][1].y, v[u][1].z, v[u][1].w};
#pragma unroll
      for (int x = 0; x < 8; ++x) {
        if (eb + x >= a.n) continue;
        f(float_to_okey(full ? fv[x] : sc[eb + x]));
      }
    }
  }
}

// `after_issue` runs once, after the first sample loads are issued (the caller's
// own loads then queue behind them). With `refine`, the sample is read a second
// time to place the threshold inside its 12-bit digit: the digit's sampled keys
// are counted by their next 8 key bits and the threshold becomes the lower edge
// of the sub-digit holding the remaining rank, so the candidates exceed the
// target by at most 1/256 of a digit instead of a whole digit.
template <typename F>
__device__ uint32_t row_sample_threshold_cta(const SelectArgs& a, const float* sc, SelectSmem& sm,
                                             int cshift, bool refine, F&& after_issue) {
  const int tid = threadIdx.x, lane = tid & 31;
  uint32_t* priv = reinterpret_cast<uint32_t*>(sm.buf);
  uint32_t* my_samp = priv + (lane & (kSampleCopies - 1)) * kSampleStride;
  uint32_t ns = 0;
  for_each_sample(a, sc, cshift, [&](uint32_t key) {
    atomicAdd(&my_samp[key >> 20], 1u);
    ++ns;
  }, after_issue);
  ns = __reduce_add_sync(0xffffffffu, ns);
  if (lane == 0 && ns) atomicAdd(&sm.nsamp, ns);
  __syncthreads();
  for (int i = tid; i < kSampleBins; i += kThreads) {
    uint32_t cnt = 0;
#pragma unroll
    for (int q = 0; q < kSampleCopies; ++q) cnt += priv[q * kSampleStride + i];
    sm.hist[i] = cnt;
  }
  __syncthreads();
  const double nsd = double(sm.nsamp);
  const double expect = double(a.k) * nsd / double(a.n);
  const double m = expect * 1.1 + 4.0 * sqrt(expect) + 8.0;
  if (!(m < nsd)) return 1u;  // every key
  find_bin(sm, kSampleBins, uint32_t(m));
  const uint32_t b = sm.bin;
  if (!refine) return b << 20;
  const uint32_t need = uint32_t(m) - sm.above;  // >= 1: rank m lies inside digit b
  for (int i = tid; i < 256; i += kThreads) sm.hist[i] = 0u;
  __syncthreads();
  for_each_sample(a, sc, cshift, [&](uint32_t key) {
    if ((key >> 20) == b) atomicAdd(&sm.hist[(key >> 12) & 0xffu], 1u);
  }, [] {});
  __syncthreads();
  find_bin(sm, 256, need);
  return (b << 20) | (sm.bin << 12);
}

// row_sample_threshold_cta for a row streamed by a cluster (2^8-column chunks, with
// the refinement), the sample split over the cluster: CTA `rank` counts the chunks
// g with g % kCluster == rank, the histograms are summed through distributed shared
// memory, so every CTA reaches the same threshold from a quarter of the loads.
// Cluster barriers: on entry the kernel-start arrive is outstanding; on return one
// arrive is outstanding again (the caller's next cluster_wait completes it).
__device__ uint32_t row_sample_threshold_split(const SelectArgs& a, const float* sc, SelectSmem& sm,
                                               cg::cluster_group& cluster, unsigned rank) {
  constexpr int cshift = 8;
  const int tid = threadIdx.x, lane = tid & 31;
  uint32_t* priv = reinterpret_cast<uint32_t*>(sm.buf);
  uint32_t* my_samp = priv + (lane & (kSampleCopies - 1)) * kSampleStride;
  uint32_t* tot = priv;                  // the summed histogram (the copies are summed first)
  uint32_t* tot2 = priv + kSampleBins;   // the summed refinement histogram
  uint32_t ns = 0;
  for_each_sample(a, sc, cshift, [&](uint32_t key) {
    atomicAdd(&my_samp[key >> 20], 1u);
    ++ns;
  }, [] {}, int(rank), kCluster);
  ns = __reduce_add_sync(0xffffffffu, ns);
  if (lane == 0 && ns) atomicAdd(&sm.nsamp, ns);
  __syncthreads();
  for (int i = tid; i < kSampleBins; i += kThreads) {
    uint32_t cnt = 0;
#pragma unroll
    for (int q = 0; q < kSampleCopies; ++q) cnt += priv[q * kSampleStride + i];
    sm.hist[i] = cnt;
  }
  __syncthreads();
  cluster_wait();    // the kernel-start phase: every CTA has started
  cluster_arrive();  // this CTA's partial histogram and count
  cluster_wait();
  uint32_t nsamp = 0;
#pragma unroll
  for (int r = 0; r < kCluster; ++r) nsamp += *cluster.map_shared_rank(&sm.nsamp, r);
  for (int i = tid; i < kSampleBins; i += kThreads) {
    uint32_t s = 0;
#pragma unroll
    for (int r = 0; r < kCluster; ++r) s += cluster.map_shared_rank(sm.hist, r)[i];
    tot[i] = s;
  }
  __syncthreads();
  cluster_arrive();  // done reading the peers' histograms
  const double nsd = double(nsamp);
  const double expect = double(a.k) * nsd / double(a.n);
  const double m = expect * 1.1 + 4.0 * sqrt(expect) + 8.0;
  if (!(m < nsd)) return 1u;  // every key (the same answer in every CTA)
  find_bin(sm, kSampleBins, uint32_t(m), tot);
  const uint32_t b = sm.bin;
  const uint32_t need = uint32_t(m) - sm.above;  // >= 1: rank m lies inside digit b
  cluster_wait();    // every CTA is done with the partial histograms
  for (int i = tid; i < 256; i += kThreads) sm.hist[i] = 0u;
  __syncthreads();
  for_each_sample(a, sc, cshift, [&](uint32_t key) {
    if ((key >> 20) == b) atomicAdd(&sm.hist[(key >> 12) & 0xffu], 1u);
  }, [] {}, int(rank), kCluster);
  __syncthreads();
  cluster_arrive();  // this CTA's refinement histogram
  cluster_wait();
  for (int i = tid; i < 256; i += kThreads) {
    uint32_t s = 0;
#pragma unroll
    for (int r = 0; r < kCluster; ++r) s += cluster.map_shared_rank(sm.hist, r)[i];
    tot2[i] = s;
  }
  __syncthreads();
  cluster_arrive();  // done reading (outstanding for the caller)
  find_bin(sm, 256, need, tot2);
  return (b << 20) | (sm.bin << 12);
}

// dst[0, n) = src[0, n) (global, L2) with eight loads of each thread in flight,
// every candidate also counted into its fine bin of [thr, kmax] (sm.hist zero on
// entry).
__device__ __forceinline__ void copy_in_counted(SelectSmem& sm, uint64_t* dst, const uint64_t* src,
                                                uint32_t n, uint32_t kmax, int shift) {
  for (uint32_t b = 0; b < n; b += 8 * kThreads) {
    uint64_t v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const uint32_t i = b + u * kThreads + threadIdx.x;
      v[u] = i < n ? __ldcg(src + i) : 0ull;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const uint32_t i = b + u * kThreads + threadIdx.x;
      if (i < n) {
        dst[i] = v[u];
        atomicAdd(&sm.hist[(kmax - uint32_t(v[u] >> 32)) >> shift], 1u);
      }
    }
  }
}

// Warp-aggregated slot of this thread's first hit among the CTA's candidates
// (sm.woff counts the CTA's candidates so far).
__device__ __forceinline__ uint32_t hit_slot(uint32_t hit, SelectSmem& sm) {
  const int lane = threadIdx.x & 31;
  const uint32_t mine = __popc(hit);
  uint32_t incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  const uint32_t wtot = __shfl_sync(0xffffffffu, incl, 31);
  uint32_t wbase = 0;
  if (lane == 31 && wtot) wbase = atomicAdd(&sm.woff, wtot);
  return __shfl_sync(0xffffffffu, wbase, 31) + incl - mine;
}

// Every CTA of the cluster holds all nc candidates in sm.buf (identical slots).
// Fine-bin counting sort as on the general leader path; CTA r then ranks and
// stores the whole bins that cover output positions [r*P, (r+1)*P), P = ceil(k/4).
// A straddling bin is ranked by both neighbours, which store identical values.
// Fine-bin width (as a shift of the key difference) for candidates in [thr, kmax].
__device__ __forceinline__ int fine_shift(uint32_t thr, uint32_t kmax) {
  const uint32_t range = kmax - thr;
  int shift = 0;
  while ((range >> shift) >= uint32_t(kFineBins)) ++shift;
  return shift;
}

// With `built`, sm.hist already holds the fine-bin counts of the nc candidates.
__device__ void replicated_sort_store(const SelectArgs& a, int64_t row, SelectSmem& sm,
                                      uint32_t nc, uint32_t thr, uint32_t kmax, unsigned rank,
                                      unsigned nparts = kCluster, bool built = false) {
  const int tid = threadIdx.x, lane = tid & 31;
  const int shift = fine_shift(thr, kmax);
  if (!built) {
    for (uint32_t i = tid; i < nc; i += kThreads)
      atomicAdd(&sm.hist[(kmax - uint32_t(sm.buf[i] >> 32)) >> shift], 1u);
    __syncthreads();
  }
  {
    constexpr int kPer = kFineBins / kThreads;
    uint32_t h[kPer], tot = 0, hmax = 0;
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      h[u] = sm.hist[kPer * tid + u];
      tot += h[u];
      hmax = max(hmax, h[u]);
    }
    hmax = __reduce_max_sync(0xffffffffu, hmax);
    if (lane == 0) atomicMax(&sm.big, hmax);
    uint32_t ex = block_excl_scan(tot, sm, nullptr);
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      sm.hist[kPer * tid + u] = ex;  // start of bin
      ex += h[u];
    }
  }
  __syncthreads();
  if (sm.big > uint32_t(kRankMax)) {
    if (rank == 0) {
      block_bitonic_sort(sm, int(nc));
      write_out(a, row, sm);
    }
    return;
  }
  for (uint32_t i = tid; i < nc; i += kThreads) {
    const uint32_t f = (kmax - uint32_t(sm.buf[i] >> 32)) >> shift;
    sm.perm[atomicAdd(&sm.hist[f], 1u)] = uint16_t(i);
  }
  __syncthreads();  // hist[f] is now the end of bin f
  const uint32_t kk = uint32_t(a.k);
  const uint32_t P = (kk + nparts - 1) / nparts;
  const uint32_t p0 = rank * P, p1 = min(kk, p0 + P);
  if (p0 >= p1) return;
  const uint32_t f0 = bin_of_position(sm, p0), f1 = bin_of_position(sm, p1 - 1);
  const uint32_t q0 = f0 ? sm.hist[f0 - 1] : 0u, q1 = sm.hist[f1];
  int32_t* oi = a.out_idx + row * a.k;
  float* os = a.out_scores ? a.out_scores + row * a.k : nullptr;
  const int64_t ibase = a.idx_in ? 0 : a.index_base;
  for (uint32_t q = q0 + tid; q < q1; q += kThreads) {
    const uint32_t i = sm.perm[q];
    const uint64_t x = sm.buf[i];
    const uint32_t f = (kmax - uint32_t(x >> 32)) >> shift;
    const uint32_t s = f ? sm.hist[f - 1] : 0u;
    const uint32_t e = sm.hist[f];
    uint32_t p = s;
    for (uint32_t j = s; j < e; ++j) {
      const uint32_t pj = sm.perm[j];
      const uint64_t y = sm.buf[pj];
      p += (y > x) || (y == x && pj < i);
    }
    if (p < kk) {
      oi[p] = int32_t(int64_t(~uint32_t(x)) + ibase);
      if (os) os[p] = okey_to_float(uint32_t(x >> 32));
    }
  }
}

// One row per cluster of kCluster CTAs.
//  1. Radix threshold: every CTA histograms the top 11 key bits of its columns
//     (8 private copies, one per lane & 7, against same-address atomics) and
//     stores the histogram into its slice of the leader's shared memory; the
//     leader finds the digit holding the k-th largest key and each CTA's count
//     of keys at or above it. While that digit would bring more than kCap
//     candidates, the next 11 (then 10) bits of the keys inside it are
//     histogrammed the same way. The threshold T is the lower edge of the chosen
//     digit, so exactly the keys >= T — at least k, at most kCap — are candidates.
//  2. Every CTA writes its keys >= T, packed with their indices, into its own
//     slot range of the row's candidate buffer.
//  3. The leader counting-sorts the candidates into 8192 fine bins of
//     (max_key - key); a candidate's output position is its bin's start plus the
//     number of bin members ahead of it, and the threads walk the candidates in
//     bin order so that a warp's member loads and output stores stay together.
//     A fine bin above kRankMax members switches to a bitonic sort of all
//     candidates.
// Keys are loaded once and kept in registers when the row fits one pass
// (kResident); longer rows are re-read for each histogram level and the append.
// If even whole-key ties exceed kCap, the leader runs the general path.
template <bool kResident>
__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kThreads, 1)
    select_topk_cluster_kernel(const SelectArgs a, uint64_t* __restrict__ cand_all,
                               int64_t cand_cap) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  SelectSmem& sm = *reinterpret_cast<SelectSmem*>(smem_raw);
  cg::cluster_group cluster = cg::this_cluster();
  const unsigned rank = cluster.block_rank();
  const int64_t row = blockIdx.x / kCluster;
  if (a.rows_dyn != nullptr && row >= *a.rows_dyn) return;  // the whole cluster leaves
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const float* sc = a.scores + row * a.ld;
  const int32_t* ix = a.idx_in ? a.idx_in + row * a.ld : nullptr;
  const int64_t npass = kResident ? 1 : (a.n + kPass - 1) / kPass;
  const int64_t my_base = int64_t(rank) * kThreads * kKeys;
  uint32_t* priv = reinterpret_cast<uint32_t*>(sm.buf);  // [kPriv][kPrivStride]
  uint32_t* my_priv = priv + (lane & (kPriv - 1)) * kPrivStride;
  SelectSmem* lead = cluster.map_shared_rank(&sm, 0);
  uint32_t* lead_slice = cluster.map_shared_rank(sm.hist, 0) + rank * kLevelBins;

  static_assert(kPriv * kPrivStride >= kSampleCopies * kSampleStride, "sample copies fit the private histograms");
  for (int i = tid; i < kPriv * kPrivStride; i += kThreads) priv[i] = 0u;
  if (tid == 0) {
    sm.kmax = 0;
    sm.woff = 0;
    sm.big = 0;
    sm.nsamp = 0;
  }
  if (tid < kCluster) sm.acc[tid] = 0;
  __syncthreads();
  cluster_arrive();  // every CTA has started and initialised its shared memory
  grid_dependency_wait();
  asm volatile("griddepcontrol.launch_dependents;");  // e.g. the publish of the peer exchange
  uint32_t kv[kKeys];
  float4 raw[kKeys / 4];

  {
    // ---- fast path -------------------------------------------------------------------
    // Every CTA computes the threshold T from the same row sample; its keys >= T
    // are its candidates. The CTAs tell each other their counts; when the row's
    // total is within [k, kCap], each CTA appends its candidates to its slot range
    // of the row's candidate buffer (L2), and after a cluster barrier every CTA
    // loads all of them, counting-sorts them and stores its quarter of the output.
    // Rows longer than one pass stream their keys once, appending the hits to the
    // CTA's quarter of the buffer.
    uint64_t* cand = cand_all + row * cand_cap;
    // the row's own keys are loaded (rows held in registers) while the sample is
    // counted, their loads queued behind the sample's
    uint32_t thr;
    if (kResident) {
      thr = row_sample_threshold_cta(a, sc, sm, 7, false, [&] { load_raw(sc, my_base, a.n, raw); });
    } else {
      thr = row_sample_threshold_split(a, sc, sm, cluster, rank);
    }
    const uint32_t quarter = uint32_t(cand_cap / kCluster);
    uint32_t kmx = 0;
    uint32_t hit = 0, slot0 = 0;
    if (kResident) {
      convert_raw(raw, my_base, a.n, kv);
#pragma unroll
      for (int j = 0; j < kKeys; ++j) {
        kmx = max(kmx, kv[j]);
        if (kv[j] >= thr) hit |= 1u << j;
      }
      slot0 = hit_slot(hit, sm);
    } else {
      // the stream, in half passes (16 keys per thread), software-pipelined: the
      // loads of the next half are in flight while this half is compared and its
      // hits appended
      uint64_t* mine_buf = cand + int64_t(rank) * quarter;
      const int64_t nhalf = npass * 2;
      auto load_half = [&](int64_t hh, float4 (&v)[4]) {
        const int64_t base = (hh >> 1) * kPass + my_base;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int64_t e = base + (int64_t((4 * int(hh & 1) + u) * kThreads + tid) << 2);
          if (e + 4 <= a.n) {
            v[u] = __ldcs(reinterpret_cast<const float4*>(sc + e));
          } else {
            v[u].x = e + 0 < a.n ? sc[e + 0] : 0.f;
            v[u].y = e + 1 < a.n ? sc[e + 1] : 0.f;
            v[u].z = e + 2 < a.n ? sc[e + 2] : 0.f;
            v[u].w = e + 3 < a.n ? sc[e + 3] : 0.f;
          }
        }
      };
      // Keys are compared as floats: for every threshold up to +inf's order key the
      // float test equals the order-key test, except -0 against a +0 threshold, which
      // is lowered to -0 (a superset; every CTA of the row does the same). Thresholds
      // in the NaN range (rows dominated by NaN) confirm each passing key on its
      // order key. The largest key is taken over the stored hits (the fine bins span
      // [thr, largest hit]; a CTA that cannot store all its hits fails the fast path).
      if (thr == 0x80000000u) thr = 0x7fffffffu;
      const bool float_exact = thr <= 0xff800000u;
      const float thr_f = okey_to_float(thr);
      float4 nx[4];
      load_half(0, nx);
      for (int64_t hh = 0; hh < nhalf; ++hh) {
        const float4 cu[4] = {nx[0], nx[1], nx[2], nx[3]};
        if (hh + 1 < nhalf) load_half(hh + 1, nx);
        const int64_t base = (hh >> 1) * kPass + my_base;
        const int64_t cb = base + (int64_t(4 * int(hh & 1) * kThreads + tid) << 2);  // column of key 0
        const bool inside = cb + int64_t(3 * kThreads * 4 + 3) < a.n;  // every key of the half is a column
        const float fv[16] = {cu[0].x, cu[0].y, cu[0].z, cu[0].w, cu[1].x, cu[1].y, cu[1].z, cu[1].w,
                              cu[2].x, cu[2].y, cu[2].z, cu[2].w, cu[3].x, cu[3].y, cu[3].z, cu[3].w};
        uint32_t h = 0;
        if (float_exact) {
#pragma unroll
          for (int j = 0; j < 16; ++j) h |= (fv[j] < thr_f ? 0u : 1u) << j;  // NaN: a hit
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (!(fv[j] < thr_f) && float_to_okey(fv[j]) >= thr) h |= 1u << j;
        }
        if (!inside) {  // the padding past the row's end
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (cb + int64_t(j >> 2) * kThreads * 4 + (j & 3) >= a.n) h &= ~(1u << j);
        }
        if (__any_sync(0xffffffffu, h != 0u)) {
          const uint32_t slot = hit_slot(h, sm);
          if (h != 0u && slot + uint32_t(__popc(h)) <= quarter) {
            uint64_t* dst = mine_buf + slot;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              if (h & (1u << j)) {
                const int64_t col = cb + int64_t(j >> 2) * kThreads * 4 + (j & 3);
                const uint32_t key = float_to_okey(fv[j]);
                kmx = max(kmx, key);
                dst[__popc(h & ((1u << j) - 1u))] = pack_cand(key, ix ? uint32_t(ix[col]) : uint32_t(col));
              }
            }
          }
        }
      }
    }
    kmx = __reduce_max_sync(0xffffffffu, kmx);
    if (lane == 0) atomicMax(&sm.kmax, kmx);
    __syncthreads();
    // every CTA's count and largest key to every CTA (the first wait completes the
    // outstanding arrive: the kernel-start one, or the split sample's last)
    cluster_wait();
    if (tid < kCluster) {
      SelectSmem* peer = cluster.map_shared_rank(&sm, tid);
      peer->fcount[rank] = sm.woff;
      peer->fkmax[rank] = sm.kmax;
    }
    cluster_arrive();
    cluster_wait();
    uint32_t total = 0, cbase = 0, kmax = 0, most = 0;
#pragma unroll
    for (int r = 0; r < kCluster; ++r) {
      if (r < int(rank)) cbase += sm.fcount[r];
      total += sm.fcount[r];
      most = max(most, sm.fcount[r]);
      kmax = max(kmax, sm.fkmax[r]);
    }
    // the same decision in every CTA of the cluster
    if (total >= uint32_t(a.k) && total <= uint32_t(kCap) && (kResident || most <= quarter)) {
      const int shift = fine_shift(thr, kmax);
      for (int i = tid; i < kFineBins; i += kThreads) sm.hist[i] = 0u;  // the sort's fine bins
      if (tid == 0) sm.big = 0;
      if (kResident) {
        // this CTA's candidates, compacted in its candidate space first (free: the
        // sample's private histograms are summed), then stored to its slot range
        // with coalesced stores
        uint64_t* stage = sm.buf;
        const uint32_t ncta = sm.fcount[rank];
        // a hit's slot follows from the hit mask (no running count), its column
        // from the key layout
        uint64_t* dst = stage + slot0;
        const uint32_t colbase = uint32_t(my_base) + uint32_t(tid) * 4u;
        if (ix == nullptr) {
#pragma unroll
          for (int j = 0; j < kKeys; ++j)
            if (hit & (1u << j))
              dst[__popc(hit & ((1u << j) - 1u))] =
                  pack_cand(kv[j], colbase + uint32_t((j >> 2) * kThreads * 4 + (j & 3)));
        } else {
#pragma unroll
          for (int j = 0; j < kKeys; ++j)
            if (hit & (1u << j))
              dst[__popc(hit & ((1u << j) - 1u))] =
                  pack_cand(kv[j], uint32_t(ix[colbase + uint32_t((j >> 2) * kThreads * 4 + (j & 3))]));
        }
        __syncthreads();
        for (uint32_t i = tid; i < ncta; i += kThreads) cand[cbase + i] = stage[i];
        cluster_arrive();  // the candidate stores are visible to the cluster after the wait
        cluster_wait();
        copy_in_counted(sm, sm.buf, cand, total, kmax, shift);
      } else {
        __syncthreads();  // the fine bins are zero
        uint32_t off = 0;
#pragma unroll 1
        for (int r = 0; r < kCluster; ++r) {
          copy_in_counted(sm, sm.buf + off, cand + int64_t(r) * quarter, sm.fcount[r], kmax, shift);
          off += sm.fcount[r];
        }
      }
      __syncthreads();
      replicated_sort_store(a, row, sm, total, thr, kmax, rank, kCluster, true);
      return;
    }
    // the sample missed (fewer than k keys above the threshold, or more than the
    // buffer holds): the exact path below, from a clean state
    __syncthreads();
    for (int i = tid; i < kPriv * kPrivStride; i += kThreads) priv[i] = 0u;
    if (tid == 0) sm.woff = 0;
    __syncthreads();
    cluster_arrive();
  }

  // ---- 1. threshold ------------------------------------------------------------------
  uint32_t need = uint32_t(a.k), above_total = 0, pfx = 0, thr = 0, kmax_local = 0;
  bool found = false;
#pragma unroll 1
  for (int level = 0; level < 3; ++level) {
    const int dshift = level == 0 ? 21 : (level == 1 ? 10 : 0);
    const int nbits = level == 2 ? 10 : 11;
    const int pshift = level == 1 ? 21 : 10;  // prefix bits above the digit (levels 1, 2)
    const int nb = 1 << nbits;
    const uint32_t dmask = uint32_t(nb) - 1u;
    if (level > 0) {
      for (int i = tid; i < kPriv * kPrivStride; i += kThreads) priv[i] = 0u;
      __syncthreads();
    }
    auto accumulate = [&](const uint32_t (&keys)[kKeys]) {
#pragma unroll
      for (int j = 0; j < kKeys; ++j) {
        const uint32_t key = keys[j];
        const bool match = level == 0 ? key != 0u : (key >> pshift) == pfx;
        if (match) atomicAdd(&my_priv[(key >> dshift) & dmask], 1u);
        if (level == 0) kmax_local = max(kmax_local, key);
      }
    };
    if (kResident) {
      accumulate(kv);
    } else {
      for (int64_t p = 0; p < npass; ++p) {
        uint32_t kp[kKeys];
        load_keys(sc, p * kPass + my_base, a.n, kp);
        accumulate(kp);
      }
    }
    if (level == 0) {
      kmax_local = __reduce_max_sync(0xffffffffu, kmax_local);
      if (lane == 0) atomicMax(&sm.kmax, kmax_local);
    }
    __syncthreads();
    if (level == 0) cluster_wait();
    for (int i = tid; i < nb; i += kThreads) {
      uint32_t c = 0;
#pragma unroll
      for (int q = 0; q < kPriv; ++q) c += priv[q * kPrivStride + i];
      lead_slice[i] = c;
    }
    if (level == 0 && tid == 0) atomicMax(&lead->kmax, sm.kmax);
    cluster.sync();  // every CTA's histogram is in the leader's shared memory
    if (rank == 0) {
      leader_find(sm, nb, need);
      if (tid == 0) {
        // final level: CTA r's candidates are its keys above earlier digits, above
        // this digit and in it; otherwise carry the keys above this digit forward
        const bool fits = above_total + sm.above + sm.bcount <= uint32_t(kCap);
        uint32_t slot = 0;
        for (int r = 0; r < kCluster; ++r) {
          const uint32_t eq = sm.hist[r * kLevelBins + sm.bin];
          if (fits) {
            sm.base[r] = slot;
            slot += sm.acc[r] + sm.gt[r] + eq;
          } else {
            sm.acc[r] += sm.gt[r];
          }
        }
        sm.total = slot;
      }
    }
    cluster.sync();  // the leader's answer is ready
    if (tid == 0 && rank != 0) {
      sm.bin = lead->bin;
      sm.above = lead->above;
      sm.bcount = lead->bcount;
      sm.base[rank] = lead->base[rank];
    }
    __syncthreads();
    const uint32_t b = sm.bin, above = sm.above, bcount = sm.bcount;
    const uint32_t digits = (pfx << nbits) | b;
    if (above_total + above + bcount <= uint32_t(kCap)) {
      thr = digits << dshift;
      found = true;
      break;
    }
    above_total += above;
    need -= above;
    pfx = digits;
    cluster.sync();  // everyone has read the answer before the next level reuses it
  }
  if (!found) {
    if (rank == 0) select_row_general(a, row, sm);
    return;
  }

  // ---- 2. write keys >= thr into this CTA's slot range -------------------------------------
  uint64_t* cand = cand_all + row * cand_cap;
  const uint32_t cta_base = sm.base[rank];
  auto append = [&](const uint32_t (&keys)[kKeys], int64_t base) {
    uint32_t hit = 0;
#pragma unroll
    for (int j = 0; j < kKeys; ++j)
      if (keys[j] >= thr) hit |= 1u << j;
    const uint32_t mine = __popc(hit);
    uint32_t incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const uint32_t wtot = __shfl_sync(0xffffffffu, incl, 31);
    uint32_t wbase = 0;
    if (lane == 31 && wtot) wbase = atomicAdd(&sm.woff, wtot);
    wbase = __shfl_sync(0xffffffffu, wbase, 31);
    uint32_t slot = cta_base + wbase + incl - mine;
#pragma unroll
    for (int j = 0; j < kKeys; ++j) {
      if (hit & (1u << j)) {
        const int64_t col = key_column(base, j);
        const uint32_t idx = ix ? uint32_t(ix[col]) : uint32_t(col);
        if (slot < uint64_t(cand_cap)) cand[slot] = pack_cand(keys[j], idx);
        ++slot;
      }
    }
  };
  if (kResident) {
    append(kv, my_base);
  } else {
    for (int64_t p = 0; p < npass; ++p) {
      uint32_t kp[kKeys];
      load_keys(sc, p * kPass + my_base, a.n, kp);
      append(kp, p * kPass + my_base);
    }
  }
  cluster.sync();  // candidates written
  if (rank != 0) return;

  // ---- 3. leader: fine-bin counting sort, rank inside bins, permute, store ------------------
  const uint32_t nc = min(sm.total, uint32_t(cand_cap));
  for (uint32_t i = tid; i < nc; i += kThreads) sm.buf[i] = cand[i];
  for (int i = tid; i < kFineBins; i += kThreads) sm.hist[i] = 0u;
  __syncthreads();
  const uint32_t kmax = sm.kmax, range = kmax - thr;
  int shift = 0;
  while ((range >> shift) >= uint32_t(kFineBins)) ++shift;
  for (uint32_t i = tid; i < nc; i += kThreads)
    atomicAdd(&sm.hist[(kmax - uint32_t(sm.buf[i] >> 32)) >> shift], 1u);
  __syncthreads();
  {
    constexpr int kPer = kFineBins / kThreads;
    uint32_t h[kPer], tot = 0, hmax = 0;
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      h[u] = sm.hist[kPer * tid + u];
      tot += h[u];
      hmax = max(hmax, h[u]);
    }
    hmax = __reduce_max_sync(0xffffffffu, hmax);
    if (lane == 0) atomicMax(&sm.big, hmax);
    uint32_t ex = block_excl_scan(tot, sm, nullptr);
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      sm.hist[kPer * tid + u] = ex;  // start of bin
      ex += h[u];
    }
  }
  __syncthreads();
  if (sm.big > uint32_t(kRankMax)) {
    block_bitonic_sort(sm, int(nc));
    write_out(a, row, sm);
    return;
  }
  for (uint32_t i = tid; i < nc; i += kThreads) {
    const uint32_t f = (kmax - uint32_t(sm.buf[i] >> 32)) >> shift;
    sm.perm[atomicAdd(&sm.hist[f], 1u)] = uint16_t(i);
  }
  __syncthreads();  // hist[f] is now the end of bin f
  // walk the candidates in bin order: the lanes of a warp share bins, so the
  // member loads broadcast and the stores of a bin land together
  int32_t* oi = a.out_idx + row * a.k;
  float* os = a.out_scores ? a.out_scores + row * a.k : nullptr;
  const int64_t ibase = a.idx_in ? 0 : a.index_base;
  for (uint32_t q = tid; q < nc; q += kThreads) {
    const uint32_t i = sm.perm[q];
    const uint64_t x = sm.buf[i];
    const uint32_t f = (kmax - uint32_t(x >> 32)) >> shift;
    const uint32_t s = f ? sm.hist[f - 1] : 0u;
    if (s >= uint32_t(a.k)) continue;
    const uint32_t e = sm.hist[f];
    uint32_t p = s;
    for (uint32_t j = s; j < e; ++j) {
      const uint32_t pj = sm.perm[j];
      const uint64_t y = sm.buf[pj];
      p += (y > x) || (y == x && pj < i);
    }
    if (p < uint32_t(a.k)) {
      oi[p] = int32_t(int64_t(~uint32_t(x)) + ibase);
      if (os) os[p] = okey_to_float(uint32_t(x >> 32));
    }
  }
}

// One CTA per row, no cluster, for many rows: the threshold comes from a 1/16
// sample (8 consecutive columns of every 128, at a hashed offset; same rank rule
// as the cluster fast path),
// one streaming pass appends the keys >= T to shared memory, and the CTA
// counting-sorts and stores them. Rows where the sample misses (fewer than k or
// more than kCap candidates) take the general one-block path.
__global__ void __launch_bounds__(kThreads, 1) select_topk_row_kernel(const SelectArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  SelectSmem& sm = *reinterpret_cast<SelectSmem*>(smem_raw);
  const int64_t row = blockIdx.x;
  if (a.rows_dyn != nullptr && row >= *a.rows_dyn) return;
  const int tid = threadIdx.x, lane = tid & 31;
  const float* sc = a.scores + row * a.ld;
  const int32_t* ix = a.idx_in ? a.idx_in + row * a.ld : nullptr;
  uint32_t* priv = reinterpret_cast<uint32_t*>(sm.buf);
  uint32_t* my_samp = priv + (lane & (kSampleCopies - 1)) * kSampleStride;

  for (int i = tid; i < kSampleCopies * kSampleStride; i += kThreads) priv[i] = 0u;
  if (tid == 0) {
    sm.kmax = 0;
    sm.woff = 0;
    sm.big = 0;
  }
  __syncthreads();
  grid_dependency_wait();
  asm volatile("griddepcontrol.launch_dependents;");

  // ---- sample: 8 consecutive columns of every 128, at a hashed offset ----------------
  const int64_t ngroups = (a.n + 127) / 128;
  uint32_t ns = 0;
  for (int64_t g0 = 0; g0 < ngroups; g0 += int64_t(kThreads) * 4) {
    float4 v[4][2];
    int64_t e[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t g = g0 + int64_t(u) * kThreads + tid;
      e[u] = g * 128 + 8 * int64_t((uint32_t(g) * 0x9E3779B1u) >> 28);
      const bool full = g < ngroups && e[u] + 8 <= a.n;
      v[u][0] = full ? *reinterpret_cast<const float4*>(sc + e[u]) : make_float4(0.f, 0.f, 0.f, 0.f);
      v[u][1] = full ? *reinterpret_cast<const float4*>(sc + e[u] + 4) : make_float4(0.f, 0.f, 0.f, 0.f);
      if (!full) e[u] = g < ngroups ? -e[u] - 1 : INT64_MIN;  // partial or absent group
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (e[u] == INT64_MIN) continue;
      const bool full = e[u] >= 0;
      const int64_t eb = full ? e[u] : -e[u] - 1;
      const float f[8] = {v[u][0].x, v[u][0].y, v[u][0].z, v[u][0].w,
                          v[u][1].x, v[u][1].y, v[u][1].z, v[u][1].w};
#pragma unroll
      for (int x = 0; x < 8; ++x) {
        if (eb + x >= a.n) continue;
        const uint32_t key = float_to_okey(full ? f[x] : sc[eb + x]);
        atomicAdd(&my_samp[key >> 20], 1u);
        ++ns;
      }
    }
  }
  ns = __reduce_add_sync(0xffffffffu, ns);
  if (lane == 0) atomicAdd(&sm.woff, ns);  // sample count (woff is reset below)
  __syncthreads();
  for (int i = tid; i < kSampleBins; i += kThreads) {
    uint32_t cnt = 0;
#pragma unroll
    for (int q = 0; q < kSampleCopies; ++q) cnt += priv[q * kSampleStride + i];
    sm.hist[i] = cnt;
  }
  __syncthreads();
  const double nsd = double(sm.woff);
  const double expect = double(a.k) * nsd / double(a.n);
  const double m = expect * 1.1 + 4.0 * sqrt(expect) + 8.0;
  uint32_t thr = 1u;  // every key
  if (m < nsd) {
    find_bin(sm, kSampleBins, uint32_t(m));
    thr = sm.bin << 20;
  }
  __syncthreads();
  if (tid == 0) sm.woff = 0;
  __syncthreads();

  // ---- one pass: append keys >= thr ------------------------------------------------------
  uint32_t kmx = 0;
  for (int64_t base = 0; base < a.n; base += int64_t(kThreads) * kKeys) {
    uint32_t kv[kKeys];
    load_keys(sc, base, a.n, kv);
    uint32_t hit = 0;
#pragma unroll
    for (int j = 0; j < kKeys; ++j) {
      kmx = max(kmx, kv[j]);
      if (kv[j] >= thr) hit |= 1u << j;
    }
    const uint32_t mine = __popc(hit);
    uint32_t incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const uint32_t wtot = __shfl_sync(0xffffffffu, incl, 31);
    uint32_t wbase = 0;
    if (lane == 31 && wtot) wbase = atomicAdd(&sm.woff, wtot);
    uint32_t slot = __shfl_sync(0xffffffffu, wbase, 31) + incl - mine;
#pragma unroll
    for (int j = 0; j < kKeys; ++j) {
      if (hit & (1u << j)) {
        if (slot < uint32_t(kCap)) {
          const int64_t col = key_column(base, j);
          sm.buf[slot] = pack_cand(kv[j], ix ? uint32_t(ix[col]) : uint32_t(col));
        }
        ++slot;
      }
    }
  }
  kmx = __reduce_max_sync(0xffffffffu, kmx);
  if (lane == 0) atomicMax(&sm.kmax, kmx);
  __syncthreads();
  const uint32_t total = sm.woff;
  if (total < uint32_t(a.k) || total > uint32_t(kCap)) {
    select_row_general(a, row, sm);
    return;
  }
  for (int i = tid; i < kFineBins; i += kThreads) sm.hist[i] = 0u;
  __syncthreads();
  replicated_sort_store(a, row, sm, total, thr, sm.kmax, 0, 1);
}

// ---- top-k of the union of sorted runs (the sharded path's merge) --------------------
// Run r is int32 [2, rows, run_len] at rs.run[r]: a plane of fp32 score bits and a
// plane of global indices, each row sorted by descending score then ascending
// index (what every rank's prism_einsum_topk returns); the runs may sit in other
// GPUs' memory (peer-mapped exchange buffers). Candidates are compared as
// (key << 32) | ~index. A summary of every run — its entries at positions s-1,
// 2s-1, ... with s = max(1, k / 128) — bounds from below how many of its entries
// are at or above a value (s per summary entry at or above it). The threshold T is
// the largest summary entry whose bound, summed over the runs, reaches k: the
// global k-th candidate is at or above T, and fewer than k + (N + 1) s candidates
// are, however the top keys are split over the runs. Each run's entries before its
// first summary entry below T (its prefix at or above T and at most s - 1 more, which
// rank after position k; the same bound holds) are staged in shared memory (sized
// on the host for that bound) and merged pairwise by a
// merge-path tree (ties between equal candidates: lower run first), or, where two
// tree buffers do not fit, every staged candidate is ranked by binary searches in
// the other runs' prefixes; the candidates ranked below k are the output. If ties
// at T make the prefixes exceed the staging, the binary searches run in global
// memory instead (slow, same result).
//
// Few rows: a cluster of 4 CTAs of 1024 threads per row (each stages a quarter and
// makes a quarter of the result). More rows than a wave of such clusters: one CTA
// of 256 threads per row, several per SM, so that every row runs at once.
constexpr int kMergeMaxRuns = kMergeRunsMax;
constexpr int kMergeSumm = 128;
constexpr int kMergeMaxSmem = 227 * 1024;  // dynamic shared memory of one merge CTA, at most

struct MergeShared {
  uint32_t rlen[kMergeMaxRuns + 1], roff[kMergeMaxRuns + 1];  // prefix length, staging offset
  unsigned long long rthr;                                      // threshold candidate
  const int32_t* runs[kMergeMaxRuns];                           // the run pointers
};

__device__ __forceinline__ uint64_t run_cand(const int32_t* const* runs, int r, int64_t rows,
                                             int64_t row, int64_t run_len, int64_t j) {
  const int32_t* s = runs[r] + row * run_len + j;
  return (uint64_t(float_to_okey(__int_as_float(s[0]))) << 32) | uint64_t(~uint32_t(s[rows * run_len]));
}

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Spins until *p == want or timeout_ns of %globaltimer pass (false).
__device__ bool wait_flag_eq(const uint64_t* p, uint64_t want, int64_t timeout_ns) {
  const uint64_t t0 = globaltimer_ns();
  while (ld_acquire_sys(p) != want) {
    if (int64_t(globaltimer_ns() - t0) > timeout_ns) return false;
    __nanosleep(64);
  }
  return true;
}

// ---- merge-path tree over the staged prefixes ----------------------------------
// The staged prefixes of the runs lie back to back (run r at roff[r]); every
// level merges adjacent lists pairwise into the other buffer at the same
// offsets (list m of level l + 1 = runs [m 2^(l+1), (m+1) 2^(l+1))). A thread
// takes an even share of a level's output positions, finds where its first
// position splits the two inputs (the co-rank: a binary search along the merge
// path) and merges sequentially from there. Equal keys: the lower run first,
// i.e. the first input of a pair. The last level writes only the output
// positions below k of this CTA's share straight to the result.
// Merged positions [d0, d1) of X[0, a) and Y[0, b) (both descending): emit(d, key).
template <typename Emit>
__device__ __forceinline__ void merge_path_range(const uint64_t* X, uint32_t a, const uint64_t* Y, uint32_t b,
                                                 uint32_t d0, uint32_t d1, Emit&& emit) {
  uint32_t lo = d0 > b ? d0 - b : 0u, hi = d0 < a ? d0 : a;
  while (lo < hi) {  // the number of X entries among the first d0 outputs
    const uint32_t mid = (lo + hi) >> 1;
    if (X[mid] >= Y[d0 - mid - 1]) lo = mid + 1;
    else hi = mid;
  }
  uint32_t i = lo, j = d0 - lo;
  uint64_t xv = i < a ? X[i] : 0ull, yv = j < b ? Y[j] : 0ull;
  for (uint32_t d = d0; d < d1; ++d) {
    const bool take_x = j >= b || (i < a && xv >= yv);
    emit(d, take_x ? xv : yv);
    if (take_x) {
      ++i;
      xv = i < a ? X[i] : 0ull;
    } else {
      ++j;
      yv = j < b ? Y[j] : 0ull;
    }
  }
}

// Runs the levels on the staged prefixes (in buffer A = bufs[0, cap); buffer B =
// bufs[cap, 2 cap), used when there are more than two runs or stage_out is set) and
// writes result positions [p0, p1) of the row: with stage_out the last level is
// merged into shared memory too and stored with coalesced stores, else each thread
// stores its run of consecutive positions as it merges them.
template <int kT>
__device__ void merge_tree(uint64_t* bufs, uint32_t cap, const uint32_t* roff, int nruns, uint32_t total,
                           uint32_t p0, uint32_t p1, int32_t* oi, float* os, bool stage_out) {
  const int tid = threadIdx.x;
  int levels = 0;
  while ((1 << levels) < nruns) ++levels;
  uint64_t* src = bufs;
  uint64_t* dst = bufs + cap;
  auto to_result = [&](uint32_t d, uint64_t x) {
    oi[d] = int32_t(~uint32_t(x));
    if (os) os[d] = okey_to_float(uint32_t(x >> 32));
  };
  if (levels == 0) {
    for (uint32_t d = p0 + tid; d < p1; d += kT) to_result(d, src[d]);
    return;
  }
  for (int l = 0; l < levels; ++l) {
    const bool last = l == levels - 1;
    const uint32_t s0 = last ? p0 : 0u, s1 = last ? p1 : total;  // positions of this level to make
    const uint32_t per = (s1 - s0 + kT - 1) / kT;
    uint32_t pos = s0 + min(s1 - s0, per * uint32_t(tid));
    const uint32_t end = min(s1, pos + per);
    while (pos < end) {
      int m = 0;  // the pair (list of level l + 1) holding position pos
      while (((m + 1) << (l + 1)) < nruns && roff[(m + 1) << (l + 1)] <= pos) ++m;
      const int x0 = m << (l + 1);
      const int x1 = min(x0 + (1 << l), nruns), y1 = min(x0 + (2 << l), nruns);
      const uint32_t po = roff[x0], a = roff[x1] - po, b = roff[y1] - roff[x1];
      const uint32_t seg = min(end, po + a + b);
      if (last && !stage_out) {
        merge_path_range(src + po, a, src + po + a, b, pos - po, seg - po,
                         [&](uint32_t d, uint64_t x) { to_result(po + d, x); });
      } else {
        uint64_t* out = dst + po;
        merge_path_range(src + po, a, src + po + a, b, pos - po, seg - po,
                         [&](uint32_t d, uint64_t x) { out[d] = x; });
      }
      pos = seg;
    }
    __syncthreads();
    uint64_t* t = src;
    src = dst;
    dst = t;
  }
  // the last level merged into shared memory: its positions go out coalesced
  if (stage_out)
    for (uint32_t d = p0 + tid; d < p1; d += kT) to_result(d, src[d]);
}

// summ: [nruns][kMergeSumm] summary entries; buf: the staging of cap entries (tree 2:
// two buffers of cap entries; tree 1: one; tree 0: cap entries and their cap 4-byte
// score keys, ranked by binary searches).
template <int kT, int kParts>
__device__ void merge_row(const int32_t* const* runs, int nruns, int64_t rows, int64_t run_len, int k,
                          int32_t* __restrict__ out_idx, float* __restrict__ out_scores, MergeShared& sm,
                          uint64_t* summ, uint64_t* buf, uint32_t cap, int tree, int64_t row,
                          unsigned part) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  auto cand_at = [&](int r, int64_t j) { return run_cand(runs, r, rows, row, run_len, j); };
  auto parts_sync = [&] {  // every CTA of the row
    if constexpr (kParts > 1) cg::this_cluster().sync();
    else __syncthreads();
  };

  // ---- threshold from the run summaries ----------------------------------------------------
  const int64_t sstep = k / kMergeSumm > 1 ? k / kMergeSumm : 1;
  const int nsum = int(run_len / sstep < kMergeSumm ? run_len / sstep : kMergeSumm);
  if (tid == 0) sm.rthr = 0;
  {
    // each CTA of the row loads its share of the summary entries (scattered words,
    // which may cross the interconnect) and copies the rest from its cluster peers'
    // shared memory
    const int ns = nruns * nsum;
    const int s0 = ns * int(part) / kParts, s1 = ns * int(part + 1) / kParts;
    for (int eb = s0 + tid; eb < s1; eb += 8 * kT) {  // eight loads of each thread in flight
      uint64_t v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int e = eb + u * kT;
        if (e < s1) v[u] = cand_at(e / nsum, (int64_t(e % nsum) + 1) * sstep - 1);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int e = eb + u * kT;
        if (e < s1) summ[(e / nsum) * kMergeSumm + e % nsum] = v[u];
      }
    }
    parts_sync();
    if constexpr (kParts > 1) {
      cg::cluster_group cluster = cg::this_cluster();
      for (unsigned c = 0; c < unsigned(kParts); ++c) {
        if (c == part) continue;
        const uint64_t* src = cluster.map_shared_rank(summ, c);
        for (int e = ns * int(c) / kParts + tid; e < ns * int(c + 1) / kParts; e += kT) {
          const int at = (e / nsum) * kMergeSumm + e % nsum;
          summ[at] = src[at];
        }
      }
      cluster.sync();  // every CTA holds every summary; nobody reads a peer's copy any more
    }
  }
  {
    // the largest summary entry whose count reaches k: each thread's best, then the
    // warp's, then one shared atomic per warp
    uint64_t best = 0;
    for (int e = tid; e < nruns * nsum; e += kT) {
      const int re = e / nsum, ie = e - re * nsum;
      const uint64_t v = summ[re * kMergeSumm + ie];
      if (v <= best) continue;
      int64_t c = ie + 1;  // its own run's summary entries at or above it
      for (int q = 0; q < nruns; ++q) {
        if (q == re) continue;
        const uint64_t* sq = summ + q * kMergeSumm;
        int lo = 0, hi = nsum;  // summary entries of run q at or above v
        while (lo < hi) {
          const int mid = (lo + hi) >> 1;
          if (sq[mid] >= v) lo = mid + 1;
          else hi = mid;
        }
        c += lo;
      }
      if (c * sstep >= int64_t(k)) best = v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t u = __shfl_xor_sync(0xffffffffu, best, o);
      best = u > best ? u : best;
    }
    if (lane == 0 && best != 0) atomicMax(&sm.rthr, (unsigned long long)best);
  }
  __syncthreads();
  if (sm.rthr == 0 && warp == 0) {  // no summary reaches k: the largest last candidate
    uint64_t t = 0;
    if (lane < nruns) t = cand_at(lane, run_len - 1);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t u = __shfl_xor_sync(0xffffffffu, t, o);
      t = u > t ? u : t;
    }
    if (lane == 0) sm.rthr = t;
  }
  __syncthreads();
  const uint64_t thr = sm.rthr;
  // the staged length of each run: c summary entries >= T put the boundary of its
  // prefix at or above T in [c * sstep, (c + 1) * sstep - 1]; the whole window is
  // staged. Only a long unsummarised tail (runs longer than 128 s) is searched: warp r
  // narrows the boundary 32-fold per step
  for (int r = warp; r < nruns; r += kT / 32) {
    const uint64_t* sw = summ + r * kMergeSumm;
    int ns_ge = 0;
    for (int i = lane; i < nsum; i += 32) ns_ge += sw[i] >= thr ? 1 : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ns_ge += __shfl_xor_sync(0xffffffffu, ns_ge, o);
    int64_t lo = int64_t(ns_ge) * sstep;  // entries [0, lo) are >= T, entries [hi, run_len) are < T
    int64_t hi = ns_ge < nsum ? (int64_t(ns_ge) + 1) * sstep - 1 : run_len;
    if (hi > run_len) hi = run_len;
    if (hi - lo <= sstep) {
      // stage the whole window (no search across the interconnect): its entries below
      // T rank after position k (at least k staged entries are at or above T), and the
      // staging bound k + (N + 1) s still holds
      if (lane == 0) sm.rlen[r] = uint32_t(hi);
      continue;
    }
    if (hi - lo <= 64) {
      // the whole window in one round: entries lo + lane and lo + 32 + lane
      const int64_t p0 = lo + lane, p1 = lo + 32 + lane;
      const bool g0 = p0 < hi && cand_at(r, p0) >= thr;
      const bool g1 = p1 < hi && cand_at(r, p1) >= thr;
      lo += __popc(__ballot_sync(0xffffffffu, g0)) + __popc(__ballot_sync(0xffffffffu, g1));
      hi = lo;
    }
    while (lo < hi) {
      const int64_t step = (hi - lo + 31) / 32;
      const int64_t p = lo + int64_t(lane) * step;
      const bool ge = p < hi && cand_at(r, p) >= thr;
      const int c = __popc(__ballot_sync(0xffffffffu, ge));  // passing probes: lanes 0 .. c-1
      if (c == 0) break;
      const int64_t nhi = lo + int64_t(c) * step;
      lo = lo + int64_t(c - 1) * step + 1;
      hi = nhi < hi ? nhi : hi;
    }
    if (lane == 0) sm.rlen[r] = uint32_t(lo);
  }
  __syncthreads();
  if (tid == 0) {
    uint32_t acc = 0;
    for (int r = 0; r < nruns; ++r) {
      sm.roff[r] = acc;
      acc += sm.rlen[r];
    }
    sm.roff[nruns] = acc;
  }
  __syncthreads();
  const uint32_t total = sm.roff[nruns];
  const bool staged = total <= cap;  // the same on every CTA of the row
  if (staged) {
    // each CTA of the row loads its share of the staged entries (so each entry is
    // read once, from wherever the run lives), then copies the other shares from
    // its cluster peers' shared memory
    const uint32_t q0 = uint32_t(uint64_t(total) * part / kParts);
    const uint32_t q1 = uint32_t(uint64_t(total) * (part + 1) / kParts);
    // independent loads per thread in flight (a row's whole staging in one round
    // trip for the one-CTA rows), whichever runs they fall in
    constexpr int kStage = kT >= 1024 ? 8 : 16;
    for (uint32_t e0 = q0; e0 < q1; e0 += kStage * kT) {
      uint64_t v[kStage];
#pragma unroll
      for (int u = 0; u < kStage; ++u) {
        const uint32_t e = e0 + uint32_t(u * kT + tid);
        v[u] = 0;
        if (e < q1) {
          int r = 0;
          while (e >= sm.roff[r + 1]) ++r;
          v[u] = cand_at(r, e - sm.roff[r]);
        }
      }
#pragma unroll
      for (int u = 0; u < kStage; ++u) {
        const uint32_t e = e0 + uint32_t(u * kT + tid);
        if (e < q1) buf[e] = v[u];
      }
    }
    parts_sync();  // every share is staged
    if constexpr (kParts > 1) {
      cg::cluster_group cluster = cg::this_cluster();
      for (unsigned c = 0; c < unsigned(kParts); ++c) {
        if (c == part) continue;
        const uint64_t* src = cluster.map_shared_rank(buf, c);
        const uint32_t c1 = uint32_t(uint64_t(total) * (c + 1) / kParts);
        for (uint32_t e = uint32_t(uint64_t(total) * c / kParts) + tid; e < c1; e += kT) buf[e] = src[e];
      }
      cluster.sync();  // every CTA holds all entries; nobody reads a peer's copy any more
    }
    if (tree) {
      // this CTA makes its share of the k result positions (the last level)
      const uint32_t kk = min(uint32_t(k), total);
      merge_tree<kT>(buf, cap, sm.roff, nruns, total, uint32_t(uint64_t(kk) * part / kParts),
                     uint32_t(uint64_t(kk) * (part + 1) / kParts), out_idx + row * k,
                     out_scores ? out_scores + row * k : nullptr, tree == 2);
      return;
    }
    // the score keys alone, for the binary searches (4-byte probes; the index
    // word is read only when two score keys are equal)
    uint32_t* sk = reinterpret_cast<uint32_t*>(buf + cap);
    for (uint32_t e = tid; e < total; e += kT) sk[e] = uint32_t(buf[e] >> 32);
    __syncthreads();
  }
  // rank every prefix candidate: its position in its run plus, in every other run,
  // the entries ahead of it (ties: lower run first)
  int32_t* oi = out_idx + row * k;
  float* os = out_scores ? out_scores + row * k : nullptr;
  if (staged) {
    const uint32_t* sk = reinterpret_cast<const uint32_t*>(buf + cap);
    for (uint32_t e = part * kT + tid; e < total; e += kParts * kT) {
      int r = 0;
      while (e >= sm.roff[r + 1]) ++r;
      const uint32_t j = e - sm.roff[r];
      const uint32_t xs = sk[e], xi = uint32_t(buf[e]);
      uint32_t p = j;
      for (int q = 0; q < nruns; ++q) {
        if (q == r) continue;
        const uint32_t o = sm.roff[q];
        uint32_t lo = 0, hi = sm.rlen[q];
        while (lo < hi) {
          const uint32_t mid = (lo + hi) >> 1;
          const uint32_t vs = sk[o + mid];
          bool ahead = vs > xs;
          if (vs == xs) {
            const uint32_t vi = uint32_t(buf[o + mid]);
            ahead = vi > xi || (q < r && vi == xi);
          }
          if (ahead) lo = mid + 1;
          else hi = mid;
        }
        p += lo;
      }
      if (p < uint32_t(k)) {
        oi[p] = int32_t(~xi);
        if (os) os[p] = okey_to_float(xs);
      }
    }
    return;
  }
  for (uint32_t e = part * kT + tid; e < total; e += kParts * kT) {
    int r = 0;
    while (e >= sm.roff[r + 1]) ++r;
    const uint32_t j = e - sm.roff[r];
    const uint64_t x = cand_at(r, j);
    uint32_t p = j;
    for (int q = 0; q < nruns; ++q) {
      if (q == r) continue;
      uint32_t lo = 0, hi = sm.rlen[q];
      while (lo < hi) {
        const uint32_t mid = (lo + hi) >> 1;
        const uint64_t v = cand_at(q, mid);
        if (v > x || (q < r && v == x)) lo = mid + 1;
        else hi = mid;
      }
      p += lo;
    }
    if (p < uint32_t(k)) {
      oi[p] = int32_t(~uint32_t(x));
      if (os) os[p] = okey_to_float(uint32_t(x >> 32));
    }
  }
}

// With sync.self set, the merge is the read side of the peer exchange: every CTA
// first waits until each rank has published the current step (ready flags in
// this rank's header), and the last CTA to finish tells every rank that this
// rank has read its run (ack flags), then (wait_acks) waits until every rank has
// read this rank's run, so that the next step may overwrite it. All waits are
// bounded by sync.timeout_ns and report kStatusTimeout in this rank's header; a
// CTA whose wait expired merges whatever the buffers hold (every access stays in
// bounds, and every CTA of a cluster takes the same cluster barriers).
template <int kT, int kParts>
__global__ void __cluster_dims__(kParts, 1, 1) __launch_bounds__(kT, kT >= 1024 ? 1 : 4)
    merge_runs_kernel(const RunSet rs, int nruns, int64_t rows, int64_t run_len, int k,
                      int32_t* __restrict__ out_idx, float* __restrict__ out_scores,
                      const PeerSync sync, uint32_t cap, int tree) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __shared__ MergeShared sm;
  uint64_t* summ = reinterpret_cast<uint64_t*>(smem_raw);  // [nruns][kMergeSumm]
  uint64_t* buf = summ + nruns * kMergeSumm;
  // kParts CTAs per row: each finds the same candidates, and ranks and writes its
  // own share of them
  const int64_t row = blockIdx.x / kParts;
  const unsigned part = blockIdx.x % kParts;
  const int tid = threadIdx.x;
  if (tid < nruns) sm.runs[tid] = rs.run[tid];
  grid_dependency_wait();  // a dependent launch after the publish (peer exchange)
  PeerHeader* self = sync.self;
  uint64_t step = 0, t_start = 0;
  if (self != nullptr) {
    step = self->step;
    t_start = globaltimer_ns();
    if (tid < nruns && !wait_flag_eq(&self->ready[tid], step, sync.timeout_ns))
      set_status(&self->status, kStatusTimeout);
  }
  __syncthreads();
  if (self != nullptr && blockIdx.x == 0 && tid == 0) {
    self->t_start = t_start;
    self->t_ready = globaltimer_ns();
  }
  merge_row<kT, kParts>(sm.runs, nruns, rows, run_len, k, out_idx, out_scores, sm, summ, buf, cap, tree, row,
                        part);
  if (self == nullptr) return;
  __syncthreads();  // this CTA's reads of the runs are complete
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(&self->done, 1u) == gridDim.x - 1) {
      self->done = 0;
      const uint64_t t_merged = globaltimer_ns();
      __threadfence_system();
      for (int r = 0; r < nruns; ++r) st_release_sys(&sync.peer[r]->ack[sync.rank], step);
      if (sync.wait_acks) {
        for (int r = 0; r < nruns; ++r)
          if (!wait_flag_eq(&self->ack[r], step, sync.timeout_ns)) {
            set_status(&self->status, kStatusTimeout);
            break;
          }
      }
      // this merge's share of the time: waiting for the runs (merge CTA 0),
      // merging (until the last CTA finished), waiting for the acknowledgements
      const uint64_t t0 = self->t_start, t1 = self->t_ready, t3 = globaltimer_ns();
      self->wait_ns += t1 - t0;
      self->merge_ns += t_merged > t1 ? t_merged - t1 : 0;
      self->ack_ns += t3 - t_merged;
      self->merges += 1;
    }
  }
}

// Before this rank's next local top-k overwrites its run: waits until every rank
// has acknowledged reading the run of the current step (the acks the ranks' merges
// of that step sent). A dependent launch after the scorer, which does not touch the
// run: the wait overlaps it, then griddepcontrol.wait orders the scorer's writes
// before the selection that follows. One warp; bounded like every exchange wait.
__global__ void peer_wait_acks_kernel(const PeerSync sync, int world) {
  asm volatile("griddepcontrol.launch_dependents;");
  const uint64_t s = sync.self->step;
  if (int(threadIdx.x) < world && !wait_flag_eq(&sync.self->ack[threadIdx.x], s, sync.timeout_ns))
    set_status(&sync.self->status, kStatusTimeout);
  grid_dependency_wait();
}

// Publish side of the peer exchange: advances this rank's step and marks its run
// of that step ready in every rank's header (including its own). One warp.
__global__ void peer_publish_kernel(const PeerSync sync, int world) {
  // a dependent launch: the merge may be scheduled now; the local top-k before
  // this kernel is complete and visible after the wait
  asm volatile("griddepcontrol.launch_dependents;");
  grid_dependency_wait();
  const uint64_t s = sync.self->step + 1;
  __syncwarp();
  if (threadIdx.x == 0) sync.self->step = s;
  __threadfence_system();
  if (int(threadIdx.x) < world) st_release_sys(&sync.peer[threadIdx.x]->ready[sync.rank], s);
}

__global__ void __launch_bounds__(kThreads, 1) select_topk_general_kernel(const SelectArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  SelectSmem& sm = *reinterpret_cast<SelectSmem*>(smem_raw);
  if (a.rows_dyn != nullptr && int64_t(blockIdx.x) >= *a.rows_dyn) return;
  select_row_general(a, blockIdx.x, sm);
}

}  // namespace

int64_t select_cand_cap(int64_t n) {
  // the threshold admits at most kCap candidates (and never more than n)
  return n < kCap ? n : kCap;
}

size_t select_workspace_bytes(int64_t rows, int64_t n) {
  return size_t(rows) * size_t(select_cand_cap(n)) * sizeof(uint64_t);
}

cudaError_t launch_merge_runs(const RunSet& rs, int nruns, int64_t rows, int64_t run_len, int k,
                              int32_t* out_idx, float* out_scores, const PeerSync& sync,
                              cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  if (nruns < 1 || nruns > kMergeMaxRuns) return cudaErrorInvalidValue;
  // staging for the prefixes at or above the threshold: fewer than k + (N + 1) s
  // entries (s per summary entry), and never more than the runs hold
  const int64_t sstep = k / kMergeSumm > 1 ? k / kMergeSumm : 1;
  const int64_t bound = std::min<int64_t>(int64_t(k) + (nruns + 1) * sstep, int64_t(nruns) * run_len);
  const size_t summ = size_t(nruns) * kMergeSumm * sizeof(uint64_t);
  const size_t room = (kMergeMaxSmem - summ) / 8;  // 8-byte words left for the staging
  int dev = 0, nsm = 148;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  const bool clusters = rows * 4 <= nsm;  // a 4-CTA cluster per row fits one wave
  // The merge tree (1: each thread stores the result positions it merges; 2, one CTA
  // per row: the last level merged into shared memory too and stored coalesced, which
  // measured faster there and slower for the clusters); it wants a second buffer for
  // more than one level or for the staged last level. Else (0) the ranking by binary
  // searches: the entries and their 4-byte keys.
  const size_t words1 = size_t(bound) * (nruns > 2 ? 2 : 1);
  const int tree = (!clusters && size_t(bound) * 2 <= room) ? 2 : (words1 <= room ? 1 : 0);
  const size_t tree_words = tree == 2 ? size_t(bound) * 2 : words1;
  const uint32_t cap = tree ? uint32_t(bound) : uint32_t(std::min<size_t>(size_t(bound), room * 8 / 12));
  const size_t smem = summ + (tree ? tree_words * 8 : size_t(cap) * 12);
  // the peer merge follows the publish as a dependent launch (it reads the step
  // the publish wrote only after its griddepcontrol.wait)
  const bool pdl = sync.self != nullptr;
  if (clusters) {
    auto kern = merge_runs_kernel<1024, 4>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    return launch_maybe_dependent(kern, dim3(unsigned(rows * 4)), dim3(1024), smem, pdl, stream, rs, nruns,
                                  rows, run_len, k, out_idx, out_scores, sync, cap, int(tree));
  }
  auto kern = merge_runs_kernel<256, 1>;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  return launch_maybe_dependent(kern, dim3(unsigned(rows)), dim3(256), smem, pdl, stream, rs, nruns, rows,
                                run_len, k, out_idx, out_scores, sync, cap, int(tree));
}

cudaError_t launch_merge_runs(const int32_t* runs, int nruns, int64_t rows, int64_t run_len, int k,
                              int32_t* out_idx, float* out_scores, cudaStream_t stream) {
  if (nruns < 1 || nruns > kMergeMaxRuns) return cudaErrorInvalidValue;
  RunSet rs{};
  for (int r = 0; r < nruns; ++r) rs.run[r] = runs + int64_t(r) * 2 * rows * run_len;
  return launch_merge_runs(rs, nruns, rows, run_len, k, out_idx, out_scores, PeerSync{}, stream);
}

cudaError_t launch_peer_wait_acks(const PeerSync& sync, int world, cudaStream_t stream) {
  if (world < 1 || world > kPeerMaxRanks || sync.self == nullptr) return cudaErrorInvalidValue;
  return launch_maybe_dependent(peer_wait_acks_kernel, dim3(1), dim3(32), 0, true, stream, sync, world);
}

cudaError_t launch_peer_publish(const PeerSync& sync, int world, cudaStream_t stream) {
  if (world < 1 || world > kPeerMaxRanks || sync.self == nullptr) return cudaErrorInvalidValue;
  // a dependent launch after the local top-k
  return launch_maybe_dependent(peer_publish_kernel, dim3(1), dim3(32), 0, true, stream, sync, world);
}

cudaError_t launch_select_topk(const SelectArgs& a, void* cand_ws, cudaStream_t stream) {
  const size_t smem = sizeof(SelectSmem);
  if (a.rows <= 0) return cudaSuccess;
  if (cand_ws == nullptr) {
    cudaError_t e = cudaFuncSetAttribute(select_topk_general_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    select_topk_general_kernel<<<dim3(unsigned(a.rows)), kThreads, smem, stream>>>(a);
    return cudaGetLastError();
  }
  // A dependent launch (programmatic stream serialization): the kernel may be
  // scheduled while the scorer before it drains; it reads nothing the scorer
  // writes before its griddepcontrol.wait. Not with rows_dyn, which a kernel
  // before it writes and which is read first.
  const bool pdl = a.rows_dyn == nullptr;
  if (a.rows >= kRowKernelMinRows) {
    cudaError_t e = cudaFuncSetAttribute(select_topk_row_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    return launch_maybe_dependent(select_topk_row_kernel, dim3(unsigned(a.rows)), dim3(kThreads), smem, pdl,
                                  stream, a);
  }
  const bool resident = a.n <= kPass;
  auto kern = resident ? select_topk_cluster_kernel<true> : select_topk_cluster_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  return launch_maybe_dependent(kern, dim3(unsigned(a.rows * kCluster)), dim3(kThreads), smem, pdl, stream, a,
                                static_cast<uint64_t*>(cand_ws), select_cand_cap(a.n));
}

}  // namespace prism
