// Tensor-core (tcgen05) scorer for many query rows per KV head — the prefill
// chunk of the reference's recall (reattention_exact.py:545-569: a chunk of raw
// queries against the raw, pre-RoPE middle keys of the cache, scored by
// _dense_topk, reattention.py:486-498, with the causal visibility of the chunk).
//
// Work unit: one CTA takes 256 query rows of one (batch, KV head) — two M = 128
// tiles of the rows (g, s) of the KV head's G query heads, g-major — and streams
// that head's keys in N = 128 tiles up to the last key any of its rows can see.
//   warp 0 (one lane): TMA producer, a ring of 32 KB key tiles (two 16 KB
//     128-byte-swizzled atoms: dimensions 0-63 and 64-127);
//   warp 1: allocates 512 TMEM columns; one lane issues the MMAs: per key tile
//     and query tile, 8 tcgen05.mma kind::f16 steps (M 128, N 128, K 16) into a
//     128-column fp32 accumulator; two accumulator buffers per query tile, so the
//     MMAs of tile t + 1 overlap the epilogue of tile t;
//   warps 2-9: the epilogue, two warps per TMEM lane quadrant (one per query
//     tile): 4 x tcgen05.ld of 32 columns, release of the buffer, then the mode's
//     work on the 128 scores of the thread's query row.
// The queries are loaded once with plain 16-byte loads and written to shared
// memory in the swizzled operand layout (any strides, any Sq, rows past the end
// zero). 16-bit products are exact in the fp32 accumulator, so the scores equal
// the fp32 einsum of the oracle up to summation order.
//
// RoPE'd keys (the cache _unrotate_keys un-rotates, reattention.py:743-793, with
// undo_rotary_pos_emb, _method_base.py:336-350): unrotate_planes_kernel first
// writes each key un-rotated in fp32 and split into two 16-bit planes, hi =
// round(k) and lo = round(k - hi) (|k - hi - lo| <= 2^-17 |k|). The ring then
// carries two 32 KB items per key tile, hi and lo, and the MMA issuer adds q·lo
// into the accumulator after q·hi: 16 MMA steps per key tile and query tile.
// The rotation runs once per key, not once per CTA that reads the key.
//
// Modes (the epilogue's work):
//   kScores  writes the fp32 score matrix [rows, ld] (masked keys -inf) for the
//            selection kernels;
//   kSample  streams a strided sample of the keys (every kSampleStride-th): pass
//            1 takes each row's minimum and maximum over the first quarter of the
//            sample, pass 2 a 128-bin histogram of the whole sample between them
//            (values outside in the end bins; per-row bins in shared memory);
//            the row's threshold T is the lower edge of the bin holding sample
//            rank m = 1.1 e + 4 sqrt(e) + 8, e = k * samples / keys visible
//            (-inf when the row sees at most k keys);
//   kCand    appends every visible key with score >= T, packed as
//            (fp32 score bits << 32 | ~index), to the row's candidate list
//            [rows, cap] and stores the row's count (which may exceed cap: the
//            selection then recomputes that row exactly). Per 32 scores a thread
//            builds the bit mask of hits (a subtraction and a funnel shift each),
//            parks the 32 values in shared memory (transposed: 16-byte chunk q of
//            thread t at (q * threads + t) * 16, so a warp's stores are
//            conflict-free), and walks the set bits reading the hits back by
//            index — registers cannot be indexed, and about 3 % of the scores
//            are hits.
//
// Every mbarrier wait is bounded (2 s): on expiry the kernel records
// kStatusTimeout, the roles leave their loops, and the TMEM is still freed.
#include "common.cuh"
#include "kernels.h"
#include "rope_sincos.cuh"
#include "tc_sm100.cuh"
#include "tensor_map.h"

namespace prism {
namespace {

enum PfMode : int { kScores = 0, kSample = 1, kCand = 2 };

constexpr uint32_t kAtomBytes = 128 * 128;       // 128 rows x 128 B
constexpr uint32_t kTileBytes = 2 * kAtomBytes;  // 128 rows x 128 dims
constexpr uint32_t kAOff = 0;                    // two query tiles
constexpr uint32_t kBOff = 2 * kTileBytes;       // key stages
constexpr int kHistBins = 128;
constexpr int kHistStride = 130;                 // u16 per row: 65 words, rows in distinct banks
constexpr uint32_t kTmemCols = 512;


template <int kMode>
struct PfCfg {
  // epilogue warps per (query tile, TMEM quadrant): each takes 128 / kSplit columns
  static constexpr int kSplit = kMode == kSample ? 1 : 2;
  static constexpr int kEpiWarps = 8 * kSplit;
  static constexpr int kThreads = 64 + kEpiWarps * 32;
  static constexpr int kChunks = 4 / kSplit;  // 32-column TMEM loads per thread and tile
  static constexpr int kStages = kMode == kScores ? 4 : (kMode == kSample ? 2 : 3);
  static constexpr uint32_t kHistOff = kBOff + kStages * kTileBytes;
  static constexpr uint32_t kHistBytes =
      kMode == kSample ? 256 * kHistStride * 2
                       : (kMode == kCand ? kEpiWarps * 32 * 32 * 4 : 0);  // 32 values per thread
  static constexpr uint32_t kBarOff = kHistOff + kHistBytes;
  static constexpr uint32_t kSmem = kBarOff + 256 + 1024;  // + alignment slack
};

struct PfBars {
  uint64_t full[4];
  uint64_t empty[4];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t done;
  uint32_t tmem_base;
};

struct PfArgs {
  const void* q;
  int B, Hq, Hkv, G, Sq;
  int64_t Sk;
  int64_t q_sb, q_sh, q_ss;
  int causal;
  int64_t causal_offset;
  float* scores;       // kScores: [B * Hq * Sq, ld]
  int64_t ld;
  float* thr;          // kSample (out) / kCand (in): [B * Hq * Sq]
  uint32_t* counts;    // kCand: [B * Hq * Sq, 2] (front and back list of each row)
  uint64_t* cand;      // kCand: [B * Hq * Sq, cap], filled from both ends
  int64_t cap;
  int topk;
  int pairs;           // CTAs per (batch, KV head)
  int parts;           // ring items per key tile: 1 (the keys), 2 (hi and lo planes)
  int kbatched;        // the key map has a batch dimension (else every batch row reads batch 0)
  int* status;
};

// Shifts the sign bit of d in at the bottom of m: m = (m << 1) | (d >> 31), one
// funnel shift.
__device__ __forceinline__ uint32_t push_sign(uint32_t m, float d) {
  uint32_t r;
  asm("shf.l.wrap.b32 %0, %1, %2, 1;" : "=r"(r) : "r"(__float_as_uint(d)), "r"(m));
  return r;
}

// flattened score row of row r (g-major) of KV head h in batch b
__device__ __forceinline__ int64_t score_row(const PfArgs& a, int b, int h, int64_t r) {
  const int64_t g = r / a.Sq, s = r - g * a.Sq;
  return (int64_t(b) * a.Hq + int64_t(h) * a.G + g) * a.Sq + s;
}

template <bool kBF16, int kMode>
__global__ void __launch_bounds__(PfCfg<kMode>::kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap kmap, const PfArgs a) {
  using Cfg = PfCfg<kMode>;
  constexpr int kStages = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t pad = ((raw_u32 + 1023u) & ~1023u) - raw_u32;
  uint8_t* smem = smem_raw + pad;
  const uint32_t sbase = raw_u32 + pad;
  PfBars* bars = reinterpret_cast<PfBars*>(smem + Cfg::kBarOff);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pair = blockIdx.x % a.pairs;
  const int bh = blockIdx.x / a.pairs;
  const int b = bh / a.Hkv, h = bh - b * a.Hkv;
  const int64_t R = int64_t(a.G) * a.Sq;  // query rows of this KV head
  const int64_t r0 = int64_t(pair) * 256;
  const int64_t r1 = r0 + 256 < R ? r0 + 256 : R;

  // keys any of the rows [r0, r1) can see
  int64_t nkeys = a.Sk;
  if (a.causal) {
    const int64_t smax = (r0 / a.Sq == (r1 - 1) / a.Sq) ? (r1 - 1) % a.Sq : a.Sq - 1;
    const int64_t lim = a.causal_offset + smax + 1;
    nkeys = lim < nkeys ? lim : nkeys;
  }
  // key tiles per pass (sample tiles in kSample) and passes
  const int64_t nitems = kMode == kSample ? (nkeys + kSampleStride - 1) / kSampleStride : nkeys;
  const int ntile = int((nitems + 127) / 128);
  // kSample: pass 1 (range) over the first quarter of the sample tiles, pass 2
  // (histogram) over all of them; tile t of the loop is sample tile tile_of(t)
  const int q1 = kMode == kSample ? (ntile + 3) / 4 : 0;
  const int nkt = ntile + q1;
  auto tile_of = [&](int t) { return t < q1 ? t : t - q1; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->tfull[i], 1);
      mbar_init(&bars->tempty[i], Cfg::kEpiWarps);
    }
    mbar_init(&bars->done, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  // queries -> swizzled operand tiles: row i of tile t, 16-byte chunk c of
  // dimensions [8c, 8c + 8) lands in atom c / 8 at row i, chunk (c % 8) ^ (i % 8)
  {
    const uint16_t* qg = static_cast<const uint16_t*>(a.q);
    for (int e = threadIdx.x; e < 256 * 16; e += Cfg::kThreads) {
      const int i = e >> 4, c = e & 15;
      const int64_t r = r0 + i;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (r < r1) {
        const int64_t g = r / a.Sq, s = r - g * a.Sq;
        const uint16_t* src = qg + int64_t(b) * a.q_sb + (int64_t(h) * a.G + g) * a.q_sh +
                              s * a.q_ss + 8 * c;
        v = *reinterpret_cast<const uint4*>(src);
      }
      const int t = i >> 7, ri = i & 127;
      const uint32_t off = kAOff + uint32_t(t) * kTileBytes + uint32_t(c >> 3) * kAtomBytes +
                           uint32_t(ri) * 128 + uint32_t(((c & 7) ^ (ri & 7)) * 16);
      *reinterpret_cast<uint4*>(smem + off) = v;
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    // ---- TMA producer ------------------------------------------------------------
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      const int kb = a.kbatched ? b : 0;
      const int nit = nkt * a.parts;  // ring items: key tile t, part p at u = t * parts + p
      for (int u = 0; u < nit; ++u) {
        const int s = u % kStages;
        if (u >= kStages &&
            !mbar_wait_bounded(&bars->empty[s], uint32_t((u / kStages - 1) & 1))) {
          set_status(a.status, kStatusTimeout);
          break;
        }
        const int t = a.parts == 1 ? u : u >> 1;
        const int hh = h * a.parts + (u - t * a.parts);  // the head's key plane
        const int tt = tile_of(t);  // tile within the pass
        mbar_arrive_expect_tx(&bars->full[s], kTileBytes);
        uint8_t* dst = smem + kBOff + uint32_t(s) * kTileBytes;
        tma_load_4d(dst, &kmap, 0, tt * 128, hh, kb, &bars->full[s], pol);
        tma_load_4d(dst + kAtomBytes, &kmap, 64, tt * 128, hh, kb, &bars->full[s], pol);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer --------------------------------------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_kind_f16(kBF16, 128, 128);
      bool ok = true;
      for (int t = 0; t < nkt && ok; ++t) {
        const int buf = t & 1;
        if (t >= 2) ok = mbar_wait_bounded(&bars->tempty[buf], uint32_t((t / 2 - 1) & 1));
        for (int part = 0; part < a.parts && ok; ++part) {
          const int u = t * a.parts + part, s = u % kStages;
          ok = mbar_wait_bounded(&bars->full[s], uint32_t((u / kStages) & 1));
          if (!ok) break;
          tc_fence_after();
          const uint32_t bsm = sbase + kBOff + uint32_t(s) * kTileBytes;
#pragma unroll
          for (int qt = 0; qt < 2; ++qt) {
            const uint32_t asm_ = sbase + kAOff + uint32_t(qt) * kTileBytes;
            const uint32_t d = tmem + uint32_t(buf) * 256 + uint32_t(qt) * 128;
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
              const uint32_t koff = uint32_t(ks >> 2) * kAtomBytes + uint32_t(ks & 3) * 32;
              tc_mma_f16(d, sw128_kmajor_desc(asm_ + koff), sw128_kmajor_desc(bsm + koff), idesc,
                         (part > 0 || ks > 0) ? 1u : 0u);
            }
          }
          tc_commit(&bars->empty[s]);
        }
        if (!ok) {
          set_status(a.status, kStatusTimeout);
          break;
        }
        tc_commit(&bars->tfull[buf]);
      }
      tc_commit(&bars->done);
      if (!mbar_wait_bounded(&bars->done, 0)) set_status(a.status, kStatusTimeout);
    }
  } else {
    // ---- epilogue ------------------------------------------------------------------
    constexpr int kCols = 128 / Cfg::kSplit;
    const int ew = warp - 2;
    const int quad = warp & 3;         // TMEM lanes [32 quad, 32 quad + 32)
    const int qt = (ew >> 2) & 1;      // query tile
    const int half = ew >> 3;          // column part: [half * kCols, +kCols) of each tile
    const int rl = qt * 128 + quad * 32 + lane;  // row within the CTA
    const int64_t r = r0 + rl;
    const bool rvalid = r < r1;
    int64_t nvis = 0, srow = 0;  // keys this row sees; its flattened score row
    if (rvalid) {
      const int64_t g = r / a.Sq, s = r - g * a.Sq;
      nvis = a.causal ? a.causal_offset + s + 1 : a.Sk;
      nvis = nvis < a.Sk ? nvis : a.Sk;
      nvis = nvis > 0 ? nvis : 0;
      srow = score_row(a, b, h, r);
    }
    // per-mode row state
    float mn = INFINITY, mx = -INFINITY, inv_w = 0.f;  // kSample
    uint16_t* hist = nullptr;  // kSample: the row's 128 bins (only this thread's)
    if (kMode == kSample) {
      hist = reinterpret_cast<uint16_t*>(smem + Cfg::kHistOff) + rl * kHistStride;
      for (int i = 0; i < kHistStride / 2; ++i) reinterpret_cast<uint32_t*>(hist)[i] = 0u;
    }
    float thr = -INFINITY;  // kCand
    uint32_t cnt = 0;
    uint64_t* cl = nullptr;
    float* stage = nullptr;
    if (kMode == kCand) {
      stage = reinterpret_cast<float*>(smem + Cfg::kHistOff) + (ew * 32 + lane) * 4;
      if (rvalid) {
        thr = a.thr[srow];
        cl = a.cand + srow * a.cap;
      }
    }
    const int64_t nsamp = (nvis + kSampleStride - 1) / kSampleStride;  // samples it sees
    for (int t = 0; t < nkt; ++t) {
      const int buf = t & 1;
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&bars->tfull[buf], uint32_t((t >> 1) & 1)))) {
        set_status(a.status, kStatusTimeout);
        break;
      }
      tc_fence_after();
      uint32_t v[Cfg::kChunks][32];
      const uint32_t taddr = tmem + (uint32_t(quad * 32) << 16) + uint32_t(buf) * 256 +
                             uint32_t(qt) * 128 + uint32_t(half * kCols);
#pragma unroll
      for (int c = 0; c < Cfg::kChunks; ++c) tmem_ld32(taddr + uint32_t(c) * 32, v[c]);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->tempty[buf]);
      if (!rvalid) continue;
      const int tt = tile_of(t);
      const int64_t j0 = int64_t(tt) * 128 + half * kCols;  // first key (sample) of this part
      if constexpr (kMode == kScores) {
        float* dst = a.scores + srow * a.ld + j0;
#pragma unroll
        for (int c = 0; c < Cfg::kChunks; ++c) {
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            const int64_t j = j0 + c * 32 + i;
            float4 o;
            o.x = j + 0 < nvis ? __uint_as_float(v[c][i + 0]) : -INFINITY;
            o.y = j + 1 < nvis ? __uint_as_float(v[c][i + 1]) : -INFINITY;
            o.z = j + 2 < nvis ? __uint_as_float(v[c][i + 2]) : -INFINITY;
            o.w = j + 3 < nvis ? __uint_as_float(v[c][i + 3]) : -INFINITY;
            if (j + 4 <= a.Sk) {
              *reinterpret_cast<float4*>(dst + c * 32 + i) = o;
            } else {
              if (j + 0 < a.Sk) dst[c * 32 + i + 0] = o.x;
              if (j + 1 < a.Sk) dst[c * 32 + i + 1] = o.y;
              if (j + 2 < a.Sk) dst[c * 32 + i + 2] = o.z;
            }
          }
        }
      } else if constexpr (kMode == kSample) {
        const int64_t lim = nsamp - j0;  // samples of this tile the row sees
        if (t < q1) {
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              if (c * 32 + i < lim) {
                const float x = __uint_as_float(v[c][i]);
                mn = fminf(mn, x);
                mx = fmaxf(mx, x);
              }
            }
          if (t == q1 - 1) inv_w = mx > mn ? float(kHistBins) / (mx - mn) : 0.f;
        } else {
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              if (c * 32 + i < lim) {
                const float x = __uint_as_float(v[c][i]);
                int bin = int((x - mn) * inv_w);
                bin = bin < 0 ? 0 : (bin > kHistBins - 1 ? kHistBins - 1 : bin);
                hist[bin] = uint16_t(hist[bin] + 1);
              }
            }
        }
      } else {  // kCand
        // half 0 fills the row's list from the front, half 1 from the back; a
        // chunk whose hits would pass the capacity writes none of them (the count
        // still grows, and the row is then recomputed exactly)
        constexpr int kQStride = Cfg::kEpiWarps * 32 * 4;  // floats between staged chunks
        const uint32_t cap = uint32_t(a.cap);
        const bool all_vis = j0 + kCols <= nvis;
#pragma unroll
        for (int c = 0; c < Cfg::kChunks; ++c) {
          // bit i of m = sign of (x_i - T), i.e. x_i < T, the values going in from
          // the last. x - T is never -0, and a NaN x gives the canonical NaN (sign
          // 0), so NaN is a hit: it ranks first.
          // Four independent chains of eight (one byte each), so the funnel shifts
          // do not wait on one another.
          uint32_t mb[4] = {0u, 0u, 0u, 0u};
#pragma unroll
          for (int i = 7; i >= 0; --i)
#pragma unroll
            for (int q = 0; q < 4; ++q) mb[q] = push_sign(mb[q], __uint_as_float(v[c][8 * q + i]) - thr);
          uint32_t m = __byte_perm(__byte_perm(mb[0], mb[1], 0x0040), __byte_perm(mb[2], mb[3], 0x0040),
                                   0x5410);
          m = ~m;  // hits
          if (!all_vis) {
            const int64_t lim = nvis - (j0 + 32 * c);
            m &= lim >= 32 ? 0xffffffffu : (lim <= 0 ? 0u : ((1u << lim) - 1u));
          }
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<uint4*>(stage + q * kQStride) =
                make_uint4(v[c][4 * q], v[c][4 * q + 1], v[c][4 * q + 2], v[c][4 * q + 3]);
          const uint32_t nh = __popc(m);
          uint32_t mm = cnt + nh <= cap ? m : 0u;
          int32_t off = half ? int32_t(cap - 1u - cnt) : int32_t(cnt);
          const int32_t dir = half ? -1 : 1;
          cnt += nh;
          const uint32_t jb = ~uint32_t(j0 + 32 * c);  // ~(jb + i) = jb - i
          while (mm) {
            const int i = __ffs(mm) - 1;
            mm &= mm - 1;
            const uint32_t xb = __float_as_uint(stage[(i >> 2) * kQStride + (i & 3)]);
            cl[off] = (uint64_t(xb) << 32) | uint64_t(jb - uint32_t(i));
            off += dir;
          }
        }
      }
    }
    if (rvalid && kMode == kSample) {
      float T = -INFINITY;
      if (nvis > a.topk && nsamp > 0) {
        const double e = double(a.topk) * double(nsamp) / double(nvis);
        const double m = 1.1 * e + 4.0 * sqrt(e) + 8.0;
        if (m < double(nsamp)) {
          if (inv_w > 0.f) {
            uint32_t acc = 0;
            int bin = kHistBins - 1;
            for (; bin > 0; --bin) {
              acc += hist[bin];
              if (double(acc) >= m) break;
            }
            const float w = (mx - mn) / float(kHistBins);
            T = mn + float(bin) * w - w * (1.0f / 1024.0f);
          } else {
            T = mn;  // every sample equal
          }
        }
      }
      a.thr[srow] = T;
    }
    if (rvalid && kMode == kCand) a.counts[2 * srow + half] = cnt;
    // kScores: keys past the last tile any row of this CTA sees are masked
    if (rvalid && kMode == kScores && half == 0) {
      float* dst = a.scores + srow * a.ld;
      for (int64_t j = int64_t(ntile) * 128; j < a.Sk; ++j) dst[j] = -INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// 16-bit hi / lo split of two fp32 values, packed (element 0 in the low half)
template <typename T>
struct Split16;
template <>
struct Split16<__nv_bfloat16> {
  __device__ __forceinline__ static void run(float x, float y, uint32_t& hi, uint32_t& lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(x - hf.x, y - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
  }
};
template <>
struct Split16<__half> {
  __device__ __forceinline__ static void run(float x, float y, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(x, y);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(x - hf.x, y - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
  }
};

// One warp per key position at a time: lane l takes the frequency pairs 2l and
// 2l + 1, i.e. dimensions {2l, 2l + 1} and {64 + 2l, 65 + 2l}; the angles
// fp32(pos) * inv_freq[i] and their sin / cos are computed once per position and
// applied to the key of every (batch, KV head). Un-rotation as in the decode
// scorers: r_i = x_i c + x_{i+64} s, r_{i+64} = x_{i+64} c - x_i s, in fp32.
template <typename T>
__global__ void __launch_bounds__(256) unrotate_planes_kernel(const DecodeArgs a, int nb) {
  const int lane = threadIdx.x & 31;
  const int64_t w0 = (int64_t(blockIdx.x) * 256 + threadIdx.x) >> 5;
  const int64_t nw = int64_t(gridDim.x) * 8;
  const float f0 = a.inv_freq[2 * lane], f1 = a.inv_freq[2 * lane + 1];
  const int64_t plane_words = int64_t(a.Sk) * 64;  // 32-bit words per plane
  const T* kbase = static_cast<const T*>(a.k);
  uint32_t* out = static_cast<uint32_t*>(a.planes);
  const int nh = nb * a.Hkv;
  for (int64_t j = w0; j < a.Sk; j += nw) {
    const float pf = static_cast<float>(a.pos_offset + j);
    float s0, c0, s1, c1;
    rope_sincos(__fmul_rn(pf, f0), s0, c0);
    rope_sincos(__fmul_rn(pf, f1), s1, c1);
#pragma unroll 4
    for (int bh = 0; bh < nh; ++bh) {
      const int b = bh / a.Hkv, h = bh - b * a.Hkv;
      const uint32_t* kr =
          reinterpret_cast<const uint32_t*>(kbase + int64_t(b) * a.k_sb + int64_t(h) * a.k_sh + j * 128);
      const uint32_t wa = __ldcs(kr + lane), wb = __ldcs(kr + 32 + lane);
      float x0, x0b, x1, x1b;
      Unpack<T>::run(wa, x0, x0b);  // dimensions 2l, 2l + 1
      Unpack<T>::run(wb, x1, x1b);  // dimensions 64 + 2l, 65 + 2l
      const float r0 = fmaf(x0, c0, x1 * s0), r0b = fmaf(x0b, c1, x1b * s1);
      const float r1 = fmaf(x1, c0, -(x0 * s0)), r1b = fmaf(x1b, c1, -(x0b * s1));
      uint32_t h0, l0, h1, l1;
      Split16<T>::run(r0, r0b, h0, l0);
      Split16<T>::run(r1, r1b, h1, l1);
      uint32_t* hi = out + int64_t(bh) * 2 * plane_words + j * 64;
      uint32_t* lo = hi + plane_words;
      hi[lane] = h0;
      hi[32 + lane] = h1;
      lo[lane] = l0;
      lo[32 + lane] = l1;
    }
  }
}

// batch rows of the planes: one set when the keys are shared across the batch
int plane_batches(const DecodeArgs& d) { return d.B > 1 && d.k_sb != 0 ? d.B : 1; }

// the key map of a launch: the keys, or (RoPE'd keys) the hi / lo planes
cudaError_t key_map(const DecodeArgs& d, int dtype, int key_stride, CUtensorMap* m, PfArgs& a) {
  if (d.inv_freq != nullptr) {
    if (d.planes == nullptr) return cudaErrorInvalidValue;
    const int nb = plane_batches(d);
    a.parts = 2;
    a.kbatched = nb > 1;
    return make_key_tensor_map_sw128(m, d.planes, dtype, nb, 2 * int64_t(d.Hkv), d.Sk,
                                     2 * int64_t(d.Hkv) * d.Sk * 128, int64_t(d.Sk) * 128, key_stride);
  }
  a.parts = 1;
  a.kbatched = d.B > 1 && d.k_sb != 0;
  return make_key_tensor_map_sw128(m, d.k, dtype, d.B, d.Hkv, d.Sk, d.k_sb, d.k_sh, key_stride);
}

PfArgs make_args(const DecodeArgs& d) {
  PfArgs a{};
  a.q = d.q;
  a.B = d.B;
  a.Hq = d.Hq;
  a.Hkv = d.Hkv;
  a.G = d.G;
  a.Sq = d.Sq;
  a.Sk = d.Sk;
  a.q_sb = d.q_sb;
  a.q_sh = d.q_sh;
  a.q_ss = d.q_ss;
  a.causal = d.causal;
  a.causal_offset = d.causal_offset;
  a.scores = d.scores;
  a.ld = d.ld;
  a.pairs = int((int64_t(d.G) * d.Sq + 255) / 256);
  a.status = d.status;
  return a;
}

template <int kMode>
cudaError_t launch_mode(const CUtensorMap& kmap, const PfArgs& a, int dtype, int64_t grid,
                        cudaStream_t stream) {
  auto kern = dtype == kBF16 ? prefill_tc_kernel<true, kMode> : prefill_tc_kernel<false, kMode>;
  constexpr uint32_t smem = PfCfg<kMode>::kSmem;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  kern<<<dim3(unsigned(grid)), PfCfg<kMode>::kThreads, smem, stream>>>(kmap, a);
  return cudaGetLastError();
}

}  // namespace

size_t rope_planes_bytes(int64_t B, int64_t Hkv, int64_t Sk) {
  return size_t(B) * size_t(Hkv) * 2 * size_t(Sk) * 128 * 2;
}

cudaError_t launch_unrotate_planes(const DecodeArgs& d, int dtype, int num_sms, cudaStream_t stream) {
  if (d.inv_freq == nullptr || d.planes == nullptr) return cudaErrorInvalidValue;
  const int64_t want = (int64_t(d.Sk) + 7) / 8;  // one warp per position
  const unsigned grid = unsigned(want < int64_t(num_sms) * 8 ? want : int64_t(num_sms) * 8);
  if (dtype == kBF16)
    unrotate_planes_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(d, plane_batches(d));
  else
    unrotate_planes_kernel<__half><<<grid, 256, 0, stream>>>(d, plane_batches(d));
  return cudaGetLastError();
}

bool prefill_tc_supported(const DecodeArgs& a) {
  return (a.inv_freq == nullptr || a.planes != nullptr) && int64_t(a.G) * a.Sq >= kPrefillMinRows &&
         (a.q_ss % 8) == 0 && (a.q_sh % 8) == 0 && (a.q_sb % 8) == 0 &&
         (reinterpret_cast<uintptr_t>(a.q) & 15u) == 0;
}

cudaError_t launch_prefill_scores_tc(const DecodeArgs& d, int dtype, cudaStream_t stream) {
  CUtensorMap kmap;
  PfArgs a = make_args(d);
  cudaError_t e = key_map(d, dtype, 1, &kmap, a);
  if (e != cudaSuccess) return e;
  return launch_mode<kScores>(kmap, a, dtype, int64_t(a.pairs) * d.B * d.Hkv, stream);
}

cudaError_t launch_prefill_threshold_tc(const DecodeArgs& d, int dtype, int topk, float* thr,
                                        cudaStream_t stream) {
  CUtensorMap smap;
  PfArgs a = make_args(d);
  cudaError_t e = key_map(d, dtype, kSampleStride, &smap, a);
  if (e != cudaSuccess) return e;
  a.thr = thr;
  a.topk = topk;
  return launch_mode<kSample>(smap, a, dtype, int64_t(a.pairs) * d.B * d.Hkv, stream);
}

cudaError_t launch_prefill_candidates_tc(const DecodeArgs& d, int dtype, const float* thr,
                                         uint32_t* counts, uint64_t* cand, int64_t cap,
                                         cudaStream_t stream) {
  CUtensorMap kmap;
  PfArgs a = make_args(d);
  cudaError_t e = key_map(d, dtype, 1, &kmap, a);
  if (e != cudaSuccess) return e;
  a.thr = const_cast<float*>(thr);
  a.counts = counts;
  a.cand = cand;
  a.cap = cap;
  return launch_mode<kCand>(kmap, a, dtype, int64_t(a.pairs) * d.B * d.Hkv, stream);
}

}  // namespace prism
