// Streaming top-k on the queries-as-M scorer (score_decode_wide.cu): many query
// rows per KV head sharing one long context — the shared-context decode of the
// reference's recall (several questions over one cache, _dense_topk,
// eval_harness/attention_methods/reattention.py:486-498, on keys un-rotated as in
// _unrotate_keys :743-793) — without writing the rows x keys score matrix.
//
//   1. threshold sample: the scorer on every 16th stage of 128 / Hkv positions,
//      its scores written compactly to [rows, ld_s];
//   2. wide_threshold_kernel, one CTA per row: the row's sampled scores counted by
//      their top 12 order-key bits; the threshold is placed at sample rank
//      m = 1.1 e + 4 sqrt(e) + 8 (e = k * samples / keys, the expected sample rank
//      of the k-th key): the digit holding rank m, then, inside it, the 8-bit
//      sub-digit holding the remaining rank (a second look at the row's samples);
//   3. the scorer's candidate pass: every visible key at or above its row's
//      threshold appended to the row's list (the tensor-core pass appends to a
//      segment per CTA, which the selection appends to the list);
//   4. the streaming selection (prefill_select.cu): each row's candidates sorted;
//      rows whose count lies outside [min(k, visible), cap] recomputed exactly
//      (any number of them: the fallback's scratch holds every row).
// The result equals the score-matrix path's: every key at or above the threshold
// is a candidate, so a row with at least k of them has its top-k among them.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace prism {
namespace {

constexpr int kWtThreads = 512;
constexpr int kWtCopies = 2;  // private histogram copies (lane & 1)
constexpr int kWtBatch = 8;   // sample loads in flight per thread

// Largest bin b of hist[0, nb) with sum(hist[b..nb)) >= need (need >= 1 and the
// total reaches it): *bin_out = b, *above_out = sum(hist[b+1..nb)).
__device__ void wt_find_bin(const uint32_t* hist, int nb, uint32_t need, uint32_t* wtot,
                            uint32_t* bin_out, uint32_t* above_out) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (nb + kWtThreads - 1) / kWtThreads;  // bins per thread, highest first
  const int hi = nb - 1 - per * tid;
  uint32_t local = 0;
  for (int u = 0; u < per; ++u)
    if (hi - u >= 0) local += hist[hi - u];
  uint32_t x = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wtot[warp] = x;
  __syncthreads();
  uint32_t wbase = 0;
  for (int w = 0; w < warp; ++w) wbase += wtot[w];
  const uint32_t excl = wbase + x - local;  // bins above this thread's
  if (excl < need && excl + local >= need) {
    uint32_t c = excl;
    for (int u = 0; u < per; ++u) {
      if (hi - u < 0) break;
      const uint32_t h = hist[hi - u];
      if (c + h >= need) {
        *bin_out = uint32_t(hi - u);
        *above_out = c;
        break;
      }
      c += h;
    }
  }
  __syncthreads();
}

// Per row, the threshold from its sample: S[row, 0 .. nvalid) (the sample columns
// whose positions lie below Sk form a prefix).
__global__ void __launch_bounds__(kWtThreads)
    wide_threshold_kernel(const float* __restrict__ S, int64_t ld_s, int64_t nvalid, int64_t Sk,
                          int k, float* __restrict__ thr) {
  __shared__ uint32_t hist[kWtCopies][4096];
  __shared__ uint32_t wtot[kWtThreads / 32];
  __shared__ uint32_t s_bin, s_above;
  grid_dependency_wait();  // a dependent launch: the sample is complete after the wait
  asm volatile("griddepcontrol.launch_dependents;");
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x;
  const float* srow = S + row * ld_s;
  for (int i = tid; i < kWtCopies * 4096; i += kWtThreads) (&hist[0][0])[i] = 0u;
  if (tid == 0) {
    s_bin = 0;
    s_above = 0;
  }
  __syncthreads();
  uint32_t* my = hist[tid & (kWtCopies - 1)];
  const int64_t n4 = nvalid >> 2;
  // every thread's 16-byte words of the sample, eight loads in flight at a time
  auto for_each_word = [&](auto&& f) {
    for (int64_t base = 0; base < n4; base += kWtBatch * kWtThreads) {
      float4 v[kWtBatch];
#pragma unroll
      for (int u = 0; u < kWtBatch; ++u) {
        const int64_t c4 = base + u * kWtThreads + tid;
        if (c4 < n4) v[u] = __ldcg(reinterpret_cast<const float4*>(srow) + c4);
      }
#pragma unroll
      for (int u = 0; u < kWtBatch; ++u)
        if (base + u * kWtThreads + tid < n4) f(v[u]);
    }
  };
  for_each_word([&](const float4& v) {
    atomicAdd(&my[float_to_okey(v.x) >> 20], 1u);
    atomicAdd(&my[float_to_okey(v.y) >> 20], 1u);
    atomicAdd(&my[float_to_okey(v.z) >> 20], 1u);
    atomicAdd(&my[float_to_okey(v.w) >> 20], 1u);
  });
  for (int64_t c = (n4 << 2) + tid; c < nvalid; c += kWtThreads) atomicAdd(&my[float_to_okey(srow[c]) >> 20], 1u);
  __syncthreads();
  for (int i = tid; i < 4096; i += kWtThreads) {
    uint32_t s = 0;
#pragma unroll
    for (int q = 0; q < kWtCopies; ++q) s += hist[q][i];
    hist[0][i] = s;
  }
  __syncthreads();
  const double nsd = double(nvalid);
  const double e = double(k) * nsd / double(Sk);
  const double m = e * 1.1 + 4.0 * sqrt(e) + 8.0;
  if (!(m < nsd)) {  // the sample cannot place it: every key is a candidate
    if (tid == 0) thr[row] = -INFINITY;
    return;
  }
  wt_find_bin(hist[0], 4096, uint32_t(m), wtot, &s_bin, &s_above);
  const uint32_t b = s_bin, need = uint32_t(m) - s_above;
  uint32_t* sub = hist[1];
  for (int i = tid; i < 256; i += kWtThreads) sub[i] = 0u;
  __syncthreads();
  for_each_word([&](const float4& v) {
    const float f[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t key = float_to_okey(f[u]);
      if ((key >> 20) == b) atomicAdd(&sub[(key >> 12) & 0xffu], 1u);
    }
  });
  for (int64_t c = (n4 << 2) + tid; c < nvalid; c += kWtThreads) {
    const uint32_t key = float_to_okey(srow[c]);
    if ((key >> 20) == b) atomicAdd(&sub[(key >> 12) & 0xffu], 1u);
  }
  __syncthreads();
  wt_find_bin(sub, 256, need, wtot, &s_bin, &s_above);
  // the float whose order key is the sub-digit's lower edge (a normal float
  // pattern: the low 12 key bits are zero)
  if (tid == 0) thr[row] = okey_to_float((b << 20) | (s_bin << 12));
}

size_t up256(size_t x) { return (x + 255) / 256 * 256; }

int64_t sample_ld(int64_t Sk) {
  // sample columns for any Hkv in {2, 4, 8}: at most ceil(ceil(Sk / Tp) / 16) * Tp
  // with Tp <= 64, rounded to 4 columns
  return ((Sk + 15) / 16 + 64 + 3) / 4 * 4;
}

size_t seg_bytes(int64_t rows) { return size_t(rows) * kWideMaxSegs * kWideSegCap * 8; }
size_t segn_bytes(int64_t rows) { return size_t(rows) * kWideMaxSegs * 4; }

}  // namespace

// the exact fallback can take every row (its scratch is rows x Sk fp32, the size
// of the score matrix the path does not write)
size_t wide_stream_workspace_bytes(int64_t rows, int64_t Sk, int topk) {
  return up256(prefill_stream_workspace_bytes(rows, Sk, topk, rows)) + up256(size_t(rows) * size_t(sample_ld(Sk)) * 4) +
         up256(seg_bytes(rows)) + segn_bytes(rows);
}

WideStreamPtrs wide_stream_ptrs(const DecodeArgs& a, int topk, void* ws) {
  const int64_t rows = int64_t(a.B) * a.Hq * a.Sq;
  WideStreamPtrs p;
  p.sb = stream_buffers(rows, a.Sk, topk, ws, rows);
  uint8_t* w = static_cast<uint8_t*>(ws) + up256(prefill_stream_workspace_bytes(rows, a.Sk, topk, rows));
  p.S = reinterpret_cast<float*>(w);
  p.ld_s = sample_ld(a.Sk);
  w += up256(size_t(rows) * size_t(p.ld_s) * 4);
  p.seg = reinterpret_cast<uint64_t*>(w);
  w += up256(seg_bytes(rows));
  p.segn = reinterpret_cast<uint32_t*>(w);
  return p;
}

cudaError_t wide_stream_threshold(const DecodeArgs& a, int dtype, int topk, void* ws, int num_sms,
                                  cudaStream_t stream) {
  const int64_t rows = int64_t(a.B) * a.Hq * a.Sq;
  const WideStreamPtrs p = wide_stream_ptrs(a, topk, ws);
  if (wide_sample_cols(a.Hkv, a.Sk) > p.ld_s) return cudaErrorInvalidValue;
  cudaError_t e = cudaMemsetAsync(p.sb.counts, 0, size_t(rows) * 2 * sizeof(uint32_t), stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(p.sb.flags, 0, 2 * sizeof(int), stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(p.segn, 0, segn_bytes(rows), stream);
  if (e != cudaSuccess) return e;
  DecodeArgs s = a;  // the sample's scores, compactly
  s.scores = p.S;
  s.ld = p.ld_s;
  e = wide_tc_supported(s) ? launch_wide_tc_sample(s, dtype, num_sms, stream)
                           : launch_wide_sample(s, dtype, num_sms, stream);
  if (e != cudaSuccess) return e;
  // sample column c holds position (c / Tp) * 16 * Tp + c % Tp: the columns below
  // Sk are the first nvalid
  const int64_t Tp = 128 / a.Hkv, span = int64_t(kWideSampleStride) * Tp;
  const int64_t last = (a.Sk - 1) / span;  // last sampled stage
  const int64_t nvalid = last * Tp + std::min<int64_t>(Tp, a.Sk - last * span);
  return launch_maybe_dependent(wide_threshold_kernel, dim3(unsigned(rows)), dim3(kWtThreads), 0, true, stream,
                                static_cast<const float*>(p.S), p.ld_s, nvalid, int64_t(a.Sk), topk, p.sb.thr);
}

cudaError_t wide_stream_candidates(const DecodeArgs& a, int dtype, int topk, void* ws, int num_sms,
                                   cudaStream_t stream) {
  const WideStreamPtrs p = wide_stream_ptrs(a, topk, ws);
  if (!wide_tc_supported(a) || 2 * num_sms > kWideMaxSegs)
    return launch_wide_candidates(a, dtype, p.sb.thr, p.sb.counts, p.sb.cand, p.sb.cap, num_sms, stream);
  return launch_wide_tc_candidates(a, dtype, p.sb.thr, p.sb.counts, p.sb.cand, p.sb.cap, p.seg, p.segn, num_sms,
                                   stream);
}

cudaError_t wide_stream_select(const DecodeArgs& a, int dtype, int topk, int64_t index_base, int32_t* out_idx,
                               float* out_scores, void* ws, cudaStream_t stream) {
  const WideStreamPtrs p = wide_stream_ptrs(a, topk, ws);
  return prefill_stream_select(a, dtype, topk, index_base, out_idx, out_scores, ws, stream,
                               int64_t(a.B) * a.Hq * a.Sq, p.seg, p.segn);
}

}  // namespace prism
