// Streaming top-k of the prefill chunk: the exact per-row selection over the
// candidates that prefill_tc.cu's kCand pass left (keys scoring at or above a
// sampled per-row threshold), so that the B * Hq * Sq x Sk score matrix is never
// written. Result: the top-k of each row sorted like torch.topk (descending
// score, ties by ascending index) — _dense_topk, reattention.py:486-498, with the
// causal mask of the chunk; a row that sees fewer than k keys continues with its
// masked keys (-inf) in ascending index order, as the score-matrix path does.
//
// prefill_select_kernel, one 256-thread CTA per row: the row's n candidates
// (packed (fp32 score bits << 32) | ~index) are loaded into shared memory as
// order-preserving score keys and index words and counting-sorted into 2048 fine bins between the
// row's largest and smallest candidate, logarithmic in the distance above the
// smallest (NaN, which ranks first, in bin 0; computed from the value, not from
// the packed key, whose spacing explodes around zero); a candidate's output position is its bin's start plus
// the number of bin members above it. Rows whose candidate count lies
// outside [min(k, visible keys), cap] (a threshold too high or too low for the
// row), or whose fine bins hold more than kRankMax members (massive ties), are
// listed for the exact fallback: all their scores recomputed on CUDA cores into
// a scratch row, the library's general selection on those rows, and a copy of
// the results into place. At most `nfall` rows per call can take the fallback
// (kFallbackRows on the prefill path; every row on the queries-as-M streaming
// path, whose workspace has room for it); more set kStatusCapacity.
#include "common.cuh"
#include "kernels.h"
#include "rope_sincos.cuh"

namespace prism {
namespace {

// threads of a selection CTA: 256 for the many rows of a prefill chunk; 512 (one per
// candidate segment) for the few rows of the queries-as-M tensor-core pass
constexpr int kPsThreads = 256;
constexpr int kPsThreadsSeg = 512;
static_assert(kWideMaxSegs == kPsThreadsSeg, "one candidate segment per thread");
constexpr int kPsBins = 2048;
constexpr int kPsRankMax = 64;
constexpr int kFallbackRows = 64;

struct PsArgs {
  uint64_t* cand;
  const uint32_t* counts;
  int64_t cap;
  int k;
  int64_t Sk;
  int Sq;
  int causal;
  int64_t causal_offset;
  int64_t index_base;
  int32_t* out_idx;
  float* out_scores;
  int* nflag;
  int32_t* flag_rows;
  int nfall;
  int* status;
  const uint64_t* seg;   // nullptr, or the candidate segments of the queries-as-M tensor-core
  const uint32_t* segn;  //   pass ([rows, kWideMaxSegs, kWideSegCap] and their counts)
};

__device__ __forceinline__ int64_t visible_keys(int64_t row, int Sq, int causal,
                                                int64_t causal_offset, int64_t Sk) {
  if (!causal) return Sk;
  const int64_t v = causal_offset + row % Sq + 1;
  return v < 0 ? 0 : (v < Sk ? v : Sk);
}

__device__ __forceinline__ void flag_row(const PsArgs& a, int64_t row) {
  const int slot = atomicAdd(a.nflag, 1);
  if (slot < a.nfall)
    a.flag_rows[slot] = int32_t(row);
  else
    set_status(a.status, kStatusCapacity);
}

// exclusive block scan of one value per thread (kT threads)
template <int kT>
__device__ __forceinline__ uint32_t ps_scan(uint32_t v, uint32_t* wtot, uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wtot[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = lane < kT / 32 ? wtot[lane] : 0u;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < kT / 32) wtot[lane] = w;
  }
  __syncthreads();
  const uint32_t r = (warp ? wtot[warp - 1] : 0u) + x - v;
  *total = wtot[kT / 32 - 1];
  __syncthreads();
  return r;
}

template <int kT>
__global__ void __launch_bounds__(kT) prefill_select_kernel(const PsArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  // candidates: score keys and index words (10 bytes per candidate with perm)
  uint32_t* keys = reinterpret_cast<uint32_t*>(smem);                      // [cap]
  uint32_t* idxw = keys + a.cap;                                           // [cap] ~index
  uint32_t* hist = idxw + a.cap;                                           // [kPsBins]
  uint16_t* perm = reinterpret_cast<uint16_t*>(hist + kPsBins);            // [cap]
  __shared__ uint32_t wtot[kT / 32];
  __shared__ uint32_t s_kmax, s_kmin, s_big;  // max / min key of the finite scores

  __shared__ uint32_t soff[kT == kPsThreadsSeg ? kWideMaxSegs : 1];  // segments: start of each
  // a dependent launch: the candidate pass's lists and counts are complete after the wait
  grid_dependency_wait();
  asm volatile("griddepcontrol.launch_dependents;");
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31;
  // the row's candidates at positions [0, n0) from the front of its list, then the
  // entries of the candidate pass's segments (nseg of them), then n1 from the back
  const uint32_t n0 = a.counts[2 * row];
  const uint32_t n1 = a.counts[2 * row + 1];
  uint32_t nseg = 0, my_seg_n = 0, my_seg_off = 0;  // this thread's segment: entries, start
  if constexpr (kT == kPsThreadsSeg) {
    if (a.seg != nullptr) {
      my_seg_n = a.segn[row * kWideMaxSegs + tid];
      my_seg_off = ps_scan<kT>(my_seg_n, wtot, &nseg);
      soff[tid] = my_seg_off;
    }
  }
  const uint32_t n = n0 + nseg + n1;
  const int64_t nvis = visible_keys(row, a.Sq, a.causal, a.causal_offset, a.Sk);
  const uint32_t keff = uint32_t(nvis < a.k ? nvis : a.k);
  int32_t* oi = a.out_idx + row * a.k;
  float* os = a.out_scores ? a.out_scores + row * a.k : nullptr;
  if (n > uint32_t(a.cap) || n < keff) {
    if (tid == 0) flag_row(a, row);
    return;
  }
  // masked keys after the visible ones (rows that see fewer than k keys)
  for (uint32_t p = keff + tid; p < uint32_t(a.k); p += kT) {
    oi[p] = int32_t(nvis + (p - keff) + a.index_base);
    if (os) os[p] = -INFINITY;
  }
  if (keff == 0) return;
  if (tid == 0) {
    s_kmax = 0u;
    s_kmin = 0xffffffffu;
    s_big = 0u;
  }
  for (int i = tid; i < kPsBins; i += kT) hist[i] = 0u;
  __syncthreads();
  uint32_t kmx = 0u, kmn = 0xffffffffu;
  auto put = [&](uint32_t i, uint64_t x) {  // candidate i into shared memory
    const uint32_t key = float_to_okey(__uint_as_float(uint32_t(x >> 32)));
    keys[i] = key;
    idxw[i] = uint32_t(x);
    if (key != 0xffffffffu) {  // NaN is binned apart
      kmx = max(kmx, key);
      kmn = min(kmn, key);
    }
  };
  const uint64_t* src = a.cand + row * a.cap;
  // cnt list entries at(i) into candidates dst0 + i, eight loads in flight per thread
  auto load_list = [&](uint32_t cnt, uint32_t dst0, auto&& at) {
    for (uint32_t i0 = tid; i0 < cnt; i0 += 8 * kT) {
      uint64_t v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const uint32_t i = i0 + uint32_t(u * kT);
        if (i < cnt) v[u] = at(i);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const uint32_t i = i0 + uint32_t(u * kT);
        if (i < cnt) put(dst0 + i, v[u]);
      }
    }
  };
  load_list(n0, 0u, [&](uint32_t i) { return src[i]; });
  load_list(n1, n0 + nseg, [&](uint32_t i) { return src[a.cap - 1 - i]; });
  if constexpr (kT == kPsThreadsSeg) if (nseg > 0) {
    // the segment of every appended entry (perm serves as the map until the sort
    // below), then the entries, eight loads in flight per thread
    for (uint32_t j = 0; j < my_seg_n; ++j) perm[my_seg_off + j] = uint16_t(tid);
    __syncthreads();
    const uint64_t* sg = a.seg + row * kWideMaxSegs * kWideSegCap;
    load_list(nseg, n0, [&](uint32_t i) {
      const uint32_t s = perm[i];
      return sg[s * kWideSegCap + (i - soff[s])];
    });
  }
  kmx = __reduce_max_sync(0xffffffffu, kmx);
  kmn = __reduce_min_sync(0xffffffffu, kmn);
  if (lane == 0) {
    atomicMax(&s_kmax, kmx);
    atomicMin(&s_kmin, kmn);
  }
  __syncthreads();
  const float fmax = okey_to_float(s_kmax), fmin = okey_to_float(s_kmin);
  // Bins logarithmic in the distance above the smallest candidate: a candidate x
  // goes to bin 2047 - floor((bits(y) - bits(c)) * 2047 / (bits(range + c) - bits(c))),
  // y = (x - fmin) + c, c = range / 64. The bit pattern of a positive float grows
  // with its value and about linearly in its log, so the bins are narrow just above
  // the threshold, where the candidates crowd (a score tail thins out roughly
  // exponentially), and wide near the top; every step is a rounded subtraction or
  // addition of a constant, so the bin never increases with the score.
  const float range = fmax - fmin;
  const float c0 = range * (1.0f / 64.0f);
  const uint32_t b0 = __float_as_uint(c0);
  const uint32_t btop = __float_as_uint(range + c0);
  uint32_t mult = 0u;  // 0: one bin (equal or non-finite candidates: the massive-tie path)
  if (range > 0.f && range <= 3.0e38f && btop > b0) {
    const double m = double(kPsBins - 1) * 4294967296.0 / double(btop - b0);
    mult = m >= 4294967295.0 ? 0xffffffffu : uint32_t(m);
  }
  // bin of a score key: monotone non-increasing in the score, NaN in bin 0
  auto bin_of = [&](uint32_t key) -> uint32_t {
    if (key == 0xffffffffu) return 0u;
    const float y = (okey_to_float(key) - fmin) + c0;
    return uint32_t(kPsBins - 1) - __umulhi(__float_as_uint(y) - b0, mult);
  };
  for (uint32_t i = tid; i < n; i += kT) atomicAdd(&hist[bin_of(keys[i])], 1u);
  __syncthreads();
  {
    constexpr int kPer = kPsBins / kT;
    uint32_t h[kPer], tot = 0, hmax = 0;
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      h[u] = hist[kPer * tid + u];
      tot += h[u];
      hmax = max(hmax, h[u]);
    }
    hmax = __reduce_max_sync(0xffffffffu, hmax);
    if (lane == 0) atomicMax(&s_big, hmax);
    uint32_t total;
    uint32_t ex = ps_scan<kT>(tot, wtot, &total);
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      hist[kPer * tid + u] = ex;  // start of bin
      ex += h[u];
    }
  }
  __syncthreads();
  if (s_big > uint32_t(kPsRankMax)) {  // massive ties: exact recompute of the row
    if (tid == 0) flag_row(a, row);
    return;
  }
  for (uint32_t i = tid; i < n; i += kT) perm[atomicAdd(&hist[bin_of(keys[i])], 1u)] = uint16_t(i);
  __syncthreads();  // hist[f] is now the end of bin f
  // candidates in the bins that hold output positions [0, keff)
  uint32_t fend = 0;  // first bin whose start is >= keff
  {
    uint32_t lo = 0, hi = kPsBins;  // smallest f with end(f) >= keff
    while (lo < hi) {
      const uint32_t mid = (lo + hi) >> 1;
      if (hist[mid] >= keff) hi = mid; else lo = mid + 1;
    }
    fend = lo;
  }
  const uint32_t qend = hist[fend < kPsBins ? fend : kPsBins - 1];
  for (uint32_t q = tid; q < qend; q += kT) {
    const uint32_t i = perm[q];
    const uint32_t kx = keys[i];
    const uint32_t f = bin_of(kx);
    const uint32_t s = f ? hist[f - 1] : 0u;
    const uint32_t e = hist[f];
    uint32_t p = s, ties = 0;
    for (uint32_t j = s; j < e; ++j) {
      const uint32_t ky = keys[perm[j]];
      p += ky > kx;
      ties += ky == kx;  // this candidate included
    }
    const uint32_t xi = idxw[i];  // ~index
    if (ties > 1) {  // equal scores: the lower index goes first
      for (uint32_t j = s; j < e; ++j) {
        const uint32_t pj = perm[j];
        if (pj != i && keys[pj] == kx) p += idxw[pj] > xi;  // lower index
      }
    }
    if (p < keff) {
      oi[p] = int32_t(int64_t(~xi) + a.index_base);
      if (os) os[p] = okey_to_float(kx);
    }
  }
}

// Exact scores of the listed rows (CUDA cores): scratch[slot, j] for every key j
// (masked keys -inf). Block 0 also publishes the number of listed rows it will
// serve (min(nflag, nfall)).
template <typename T>
__global__ void __launch_bounds__(256)
    fallback_scores_kernel(const DecodeArgs a, const int* nflag, const int32_t* flag_rows,
                           int nfall, int* nserve, float* scratch) {
  __shared__ float qs[128];
  grid_dependency_wait();  // a dependent launch: the listed rows are complete after the wait
  asm volatile("griddepcontrol.launch_dependents;");
  const int nf = *nflag < nfall ? *nflag : nfall;
  if (blockIdx.x == 0 && threadIdx.x == 0) *nserve = nf;
  const int slot = blockIdx.x;
  if (slot >= nf) return;
  const int64_t row = flag_rows[slot];
  const int s = int(row % a.Sq);
  const int64_t bhq = row / a.Sq;
  const int hq = int(bhq % a.Hq), b = int(bhq / a.Hq);
  const int kvh = hq / a.G;
  const T* qr = static_cast<const T*>(a.q) + int64_t(b) * a.q_sb + int64_t(hq) * a.q_sh +
                int64_t(s) * a.q_ss;
  if (threadIdx.x < 128) qs[threadIdx.x] = to_f32<T>(qr[threadIdx.x]);
  __syncthreads();
  int64_t nvis = a.Sk;
  if (a.causal) {
    const int64_t v = a.causal_offset + s + 1;
    nvis = v < 0 ? 0 : (v < a.Sk ? v : a.Sk);
  }
  const T* kb = static_cast<const T*>(a.k) + (a.B > 1 ? int64_t(b) * a.k_sb : 0) +
                int64_t(kvh) * a.k_sh;
  float* out = scratch + int64_t(slot) * a.ld;
  if (a.inv_freq != nullptr) {
    // RoPE'd keys: un-rotated on the fly (the fp32 angle fp32(pos) * inv_freq[i],
    // sin/cos of it, x_i c + x_{i+64} s and x_{i+64} c - x_i s), dot product in fp32
    __shared__ float invf[64];
    if (threadIdx.x < 64) invf[threadIdx.x] = a.inv_freq[threadIdx.x];
    __syncthreads();
    for (int64_t j = threadIdx.x; j < a.Sk; j += 256) {
      if (j >= nvis) {
        out[j] = -INFINITY;
        continue;
      }
      const T* kr = kb + j * 128;
      const float pf = static_cast<float>(a.pos_offset + j);
      float acc = 0.f;
      for (int i = 0; i < 64; ++i) {
        float sv, cv;
        rope_sincos(__fmul_rn(pf, invf[i]), sv, cv);
        const float x0 = to_f32<T>(kr[i]), x1 = to_f32<T>(kr[i + 64]);
        acc = fmaf(qs[i], fmaf(x0, cv, x1 * sv), acc);
        acc = fmaf(qs[i + 64], fmaf(x1, cv, -(x0 * sv)), acc);
      }
      out[j] = acc;
    }
    return;
  }
  for (int64_t j = threadIdx.x; j < a.Sk; j += 256) {
    if (j >= nvis) {
      out[j] = -INFINITY;
      continue;
    }
    const uint4* kr = reinterpret_cast<const uint4*>(kb + j * 128);
    float acc = 0.f;
#pragma unroll 4
    for (int c = 0; c < 16; ++c) {
      const uint4 u = kr[c];
      float x0, x1, x2, x3, x4, x5, x6, x7;
      Unpack<T>::run(u.x, x0, x1);
      Unpack<T>::run(u.y, x2, x3);
      Unpack<T>::run(u.z, x4, x5);
      Unpack<T>::run(u.w, x6, x7);
      const float* qq = qs + 8 * c;
      acc = fmaf(qq[0], x0, acc);
      acc = fmaf(qq[1], x1, acc);
      acc = fmaf(qq[2], x2, acc);
      acc = fmaf(qq[3], x3, acc);
      acc = fmaf(qq[4], x4, acc);
      acc = fmaf(qq[5], x5, acc);
      acc = fmaf(qq[6], x6, acc);
      acc = fmaf(qq[7], x7, acc);
    }
    out[j] = acc;
  }
}

__global__ void fallback_scatter_kernel(const int* nserve, const int32_t* flag_rows, int k,
                                        const int32_t* cidx, const float* csc, int32_t* out_idx,
                                        float* out_scores) {
  grid_dependency_wait();  // a dependent launch: the fallback's selection is complete after the wait
  const int slot = blockIdx.x;
  if (slot >= *nserve) return;
  const int64_t row = flag_rows[slot];
  for (int p = threadIdx.x; p < k; p += blockDim.x) {
    out_idx[row * k + p] = cidx[int64_t(slot) * k + p];
    if (out_scores) out_scores[row * k + p] = csc[int64_t(slot) * k + p];
  }
}

size_t up256(size_t x) { return (x + 255) / 256 * 256; }

struct PsLayout {
  size_t thr, counts, cand, flags, flag_rows, scratch, sel_ws, cidx, csc, total;
};

PsLayout ps_layout(int64_t rows, int64_t Sk, int topk, int64_t nfall) {
  PsLayout L{};
  const int64_t cap = prefill_cand_cap(Sk, topk);
  const int64_t ld = (Sk + 3) / 4 * 4;
  size_t o = 0;
  L.thr = o;
  o += up256(size_t(rows) * 4);
  L.counts = o;
  o += up256(size_t(rows) * 8);
  L.cand = o;
  o += up256(size_t(rows) * size_t(cap) * 8);
  L.flags = o;  // nflag, nserve
  o += 256;
  L.flag_rows = o;
  o += up256(size_t(nfall) * 4);
  L.scratch = o;
  o += up256(size_t(nfall) * size_t(ld) * 4);
  L.sel_ws = o;
  o += up256(select_workspace_bytes(nfall, Sk));
  L.cidx = o;
  o += up256(size_t(nfall) * size_t(topk) * 4);
  L.csc = o;
  o += up256(size_t(nfall) * size_t(topk) * 4);
  L.total = o;
  return L;
}

}  // namespace

int64_t prefill_cand_cap(int64_t Sk, int topk) {
  const int64_t c = 2 * int64_t(topk) + 2048;
  return c < Sk ? c : Sk;
}

size_t prefill_stream_workspace_bytes(int64_t rows, int64_t Sk, int topk, int64_t nfall) {
  return ps_layout(rows, Sk, topk, nfall < 0 ? kFallbackRows : nfall).total;
}

namespace {
struct PsPtrs {
  float* thr;
  uint32_t* counts;
  uint64_t* cand;
  int* nflag;
  int* nserve;
  int32_t* flag_rows;
  float* scratch;
  void* sel_ws;
  int32_t* cidx;
  float* csc;
  int64_t cap;
};
PsPtrs ps_ptrs(const DecodeArgs& d, int topk, void* ws, int64_t nfall) {
  const int64_t rows = int64_t(d.B) * d.Hq * d.Sq;
  const PsLayout L = ps_layout(rows, d.Sk, topk, nfall);
  uint8_t* w = static_cast<uint8_t*>(ws);
  PsPtrs p;
  p.thr = reinterpret_cast<float*>(w + L.thr);
  p.counts = reinterpret_cast<uint32_t*>(w + L.counts);
  p.cand = reinterpret_cast<uint64_t*>(w + L.cand);
  p.nflag = reinterpret_cast<int*>(w + L.flags);
  p.nserve = p.nflag + 1;
  p.flag_rows = reinterpret_cast<int32_t*>(w + L.flag_rows);
  p.scratch = reinterpret_cast<float*>(w + L.scratch);
  p.sel_ws = w + L.sel_ws;
  p.cidx = reinterpret_cast<int32_t*>(w + L.cidx);
  p.csc = reinterpret_cast<float*>(w + L.csc);
  p.cap = prefill_cand_cap(d.Sk, topk);
  return p;
}
}  // namespace

StreamBuffers stream_buffers(int64_t rows, int64_t Sk, int topk, void* ws, int64_t nfall) {
  const PsLayout L = ps_layout(rows, Sk, topk, nfall);
  uint8_t* w = static_cast<uint8_t*>(ws);
  StreamBuffers s;
  s.thr = reinterpret_cast<float*>(w + L.thr);
  s.counts = reinterpret_cast<uint32_t*>(w + L.counts);
  s.cand = reinterpret_cast<uint64_t*>(w + L.cand);
  s.cap = prefill_cand_cap(Sk, topk);
  s.flags = reinterpret_cast<int*>(w + L.flags);
  return s;
}

cudaError_t prefill_stream_threshold(const DecodeArgs& d, int dtype, int topk, void* ws,
                                     cudaStream_t stream) {
  const PsPtrs p = ps_ptrs(d, topk, ws, kFallbackRows);
  cudaError_t e = cudaMemsetAsync(p.nflag, 0, 2 * sizeof(int), stream);
  if (e != cudaSuccess) return e;
  return launch_prefill_threshold_tc(d, dtype, topk, p.thr, stream);
}

cudaError_t prefill_stream_candidates(const DecodeArgs& d, int dtype, int topk, void* ws,
                                      cudaStream_t stream) {
  const PsPtrs p = ps_ptrs(d, topk, ws, kFallbackRows);
  return launch_prefill_candidates_tc(d, dtype, p.thr, p.counts, p.cand, p.cap, stream);
}

cudaError_t prefill_stream_select(const DecodeArgs& d, int dtype, int topk, int64_t index_base,
                                  int32_t* out_idx, float* out_scores, void* ws,
                                  cudaStream_t stream, int64_t nfall_in, const uint64_t* seg,
                                  const uint32_t* segn) {
  const int64_t nfall = nfall_in < 0 ? kFallbackRows : nfall_in;
  const PsPtrs w = ps_ptrs(d, topk, ws, nfall);
  const int64_t rows = int64_t(d.B) * d.Hq * d.Sq;
  PsArgs p{};
  p.cand = w.cand;
  p.counts = w.counts;
  p.cap = w.cap;
  p.k = topk;
  p.Sk = d.Sk;
  p.Sq = d.Sq;
  p.causal = d.causal;
  p.causal_offset = d.causal_offset;
  p.index_base = index_base;
  p.out_idx = out_idx;
  p.out_scores = out_scores;
  p.nflag = w.nflag;
  p.flag_rows = w.flag_rows;
  p.nfall = int(nfall);
  p.status = d.status;
  p.seg = seg;
  p.segn = segn;
  const size_t smem = size_t(w.cap) * 10 + kPsBins * 4;
  const bool segs = seg != nullptr;
  auto kern = segs ? prefill_select_kernel<kPsThreadsSeg> : prefill_select_kernel<kPsThreads>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  e = launch_maybe_dependent(kern, dim3(unsigned(rows)), dim3(segs ? kPsThreadsSeg : kPsThreads), smem, true, stream,
                             p);
  if (e != cudaSuccess) return e;

  // exact fallback for the listed rows (kernels return at once when none are)
  if (dtype == kBF16)
    e = launch_maybe_dependent(fallback_scores_kernel<__nv_bfloat16>, dim3(unsigned(nfall)), dim3(256), 0, true,
                               stream, d, static_cast<const int*>(w.nflag), static_cast<const int32_t*>(w.flag_rows),
                               int(nfall), w.nserve, w.scratch);
  else
    e = launch_maybe_dependent(fallback_scores_kernel<__half>, dim3(unsigned(nfall)), dim3(256), 0, true, stream, d,
                               static_cast<const int*>(w.nflag), static_cast<const int32_t*>(w.flag_rows),
                               int(nfall), w.nserve, w.scratch);
  if (e != cudaSuccess) return e;
  SelectArgs s{};
  s.scores = w.scratch;
  s.idx_in = nullptr;
  s.rows = nfall;
  s.n = d.Sk;
  s.ld = d.ld;
  s.k = topk;
  s.index_base = index_base;
  s.out_idx = w.cidx;
  s.out_scores = w.csc;
  s.status = d.status;
  s.rows_dyn = w.nserve;
  e = launch_select_topk(s, w.sel_ws, stream);
  if (e != cudaSuccess) return e;
  return launch_maybe_dependent(fallback_scatter_kernel, dim3(unsigned(nfall)), dim3(256), 0, true, stream,
                                static_cast<const int*>(w.nserve), static_cast<const int32_t*>(w.flag_rows), topk,
                                static_cast<const int32_t*>(w.cidx), static_cast<const float*>(w.csc), out_idx,
                                out_scores);
}

}  // namespace prism
