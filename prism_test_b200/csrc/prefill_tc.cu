// Tensor-core (tcgen05) scorer for many query rows per KV head — the prefill
// chunk of the reference's recall (reattention_exact.py:545-569: a chunk of raw
// queries against the raw, pre-RoPE middle keys of the cache, scored by
// _dense_topk, reattention.py:486-498, with the causal visibility of the chunk).
//
// Work unit: one CTA takes 256 query rows of one (batch, KV head) — two M = 128
// tiles of the rows (g, s) of the KV head's G query heads, g-major — and streams
// that head's keys in N = 128 tiles up to the last key any of its rows can see.
//   warp 0 (one lane): TMA producer, a 4-stage ring of 32 KB key tiles (two 16 KB
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
// Every mbarrier wait is bounded (2 s): on expiry the kernel records
// kStatusTimeout, the roles leave their loops, and the TMEM is still freed.
#include "common.cuh"
#include "kernels.h"
#include "tc_sm100.cuh"
#include "tensor_map.h"

namespace prism {
namespace {

constexpr int kPfStages = 4;
constexpr int kPfThreads = 320;
constexpr int kPfEpiWarps = 8;
constexpr uint32_t kAtomBytes = 128 * 128;       // 128 rows x 128 B
constexpr uint32_t kTileBytes = 2 * kAtomBytes;  // 128 rows x 128 dims
constexpr uint32_t kAOff = 0;                    // two query tiles
constexpr uint32_t kBOff = 2 * kTileBytes;       // key stages
constexpr uint32_t kBarOff = kBOff + kPfStages * kTileBytes;
constexpr uint32_t kPfSmem = kBarOff + 256 + 1024;  // + alignment slack
constexpr uint32_t kTmemCols = 512;

struct PfBars {
  uint64_t full[kPfStages];
  uint64_t empty[kPfStages];
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
  float* scores;  // [B * Hq * Sq, ld]
  int64_t ld;
  int pairs;      // CTAs per (batch, KV head)
  int* status;
};

// flattened score row of row r (g-major) of KV head h in batch b
__device__ __forceinline__ int64_t score_row(const PfArgs& a, int b, int h, int64_t r) {
  const int64_t g = r / a.Sq, s = r - g * a.Sq;
  return (int64_t(b) * a.Hq + int64_t(h) * a.G + g) * a.Sq + s;
}

template <bool kBF16>
__global__ void __launch_bounds__(kPfThreads, 1)
    prefill_scores_kernel(const __grid_constant__ CUtensorMap kmap, const PfArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t pad = ((raw_u32 + 1023u) & ~1023u) - raw_u32;
  uint8_t* smem = smem_raw + pad;
  const uint32_t sbase = raw_u32 + pad;
  PfBars* bars = reinterpret_cast<PfBars*>(smem + kBarOff);

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
  const int nkt = int((nkeys + 127) / 128);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPfStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->tfull[i], 1);
      mbar_init(&bars->tempty[i], kPfEpiWarps);
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
    for (int e = threadIdx.x; e < 256 * 16; e += kPfThreads) {
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
      for (int t = 0; t < nkt; ++t) {
        const int s = t % kPfStages;
        if (t >= kPfStages &&
            !mbar_wait_bounded(&bars->empty[s], uint32_t((t / kPfStages - 1) & 1))) {
          set_status(a.status, kStatusTimeout);
          break;
        }
        mbar_arrive_expect_tx(&bars->full[s], kTileBytes);
        uint8_t* dst = smem + kBOff + uint32_t(s) * kTileBytes;
        const int kb = (a.B > 1) ? b : 0;
        tma_load_4d(dst, &kmap, 0, t * 128, h, kb, &bars->full[s], pol);
        tma_load_4d(dst + kAtomBytes, &kmap, 64, t * 128, h, kb, &bars->full[s], pol);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer --------------------------------------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_kind_f16(kBF16, 128, 128);
      bool ok = true;
      for (int t = 0; t < nkt && ok; ++t) {
        const int s = t % kPfStages, buf = t & 1;
        ok = mbar_wait_bounded(&bars->full[s], uint32_t((t / kPfStages) & 1));
        if (ok && t >= 2) ok = mbar_wait_bounded(&bars->tempty[buf], uint32_t((t / 2 - 1) & 1));
        if (!ok) {
          set_status(a.status, kStatusTimeout);
          break;
        }
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
                       ks > 0 ? 1u : 0u);
          }
        }
        tc_commit(&bars->empty[s]);
        tc_commit(&bars->tfull[buf]);
      }
      tc_commit(&bars->done);
      if (!mbar_wait_bounded(&bars->done, 0)) set_status(a.status, kStatusTimeout);
    }
  } else {
    // ---- epilogue ------------------------------------------------------------------
    const int qt = (warp - 2) >> 2;      // query tile
    const int quad = warp & 3;           // TMEM lanes [32 quad, 32 quad + 32)
    const int64_t r = r0 + int64_t(qt) * 128 + quad * 32 + lane;
    const bool rvalid = r < r1;
    int64_t vis = INT64_MAX, row_off = 0;
    if (rvalid) {
      const int64_t g = r / a.Sq, s = r - g * a.Sq;
      if (a.causal) vis = a.causal_offset + s;
      row_off = score_row(a, b, h, r) * a.ld;
    }
    for (int t = 0; t < nkt; ++t) {
      const int buf = t & 1;
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&bars->tfull[buf], uint32_t((t >> 1) & 1)))) {
        set_status(a.status, kStatusTimeout);
        break;
      }
      tc_fence_after();
      uint32_t v[4][32];
      const uint32_t taddr = tmem + (uint32_t(quad * 32) << 16) + uint32_t(buf) * 256 +
                             uint32_t(qt) * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(taddr + uint32_t(c) * 32, v[c]);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->tempty[buf]);
      if (rvalid) {
        const int64_t j0 = int64_t(t) * 128;
        float* dst = a.scores + row_off + j0;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            const int64_t j = j0 + c * 32 + i;
            float4 o;
            o.x = j + 0 > vis ? -INFINITY : __uint_as_float(v[c][i + 0]);
            o.y = j + 1 > vis ? -INFINITY : __uint_as_float(v[c][i + 1]);
            o.z = j + 2 > vis ? -INFINITY : __uint_as_float(v[c][i + 2]);
            o.w = j + 3 > vis ? -INFINITY : __uint_as_float(v[c][i + 3]);
            if (j + 4 <= a.Sk) {
              *reinterpret_cast<float4*>(dst + c * 32 + i) = o;
            } else {
              if (j + 0 < a.Sk) dst[c * 32 + i + 0] = o.x;
              if (j + 1 < a.Sk) dst[c * 32 + i + 1] = o.y;
              if (j + 2 < a.Sk) dst[c * 32 + i + 2] = o.z;
            }
          }
        }
      }
    }
    // keys beyond the last visible tile are masked for every row of this CTA
    if (rvalid && a.causal) {
      for (int64_t j = int64_t(nkt) * 128; j < a.Sk; ++j) a.scores[row_off + j] = -INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

bool prefill_tc_supported(const DecodeArgs& a) {
  return a.inv_freq == nullptr && int64_t(a.G) * a.Sq >= kPrefillMinRows &&
         (a.q_ss % 8) == 0 && (a.q_sh % 8) == 0 && (a.q_sb % 8) == 0 &&
         (reinterpret_cast<uintptr_t>(a.q) & 15u) == 0;
}

cudaError_t launch_prefill_scores_tc(const DecodeArgs& d, int dtype, cudaStream_t stream) {
  CUtensorMap kmap;
  cudaError_t e = make_key_tensor_map_sw128(&kmap, d.k, dtype, d.B, d.Hkv, d.Sk, d.k_sb, d.k_sh);
  if (e != cudaSuccess) return e;
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
  const int64_t grid = int64_t(a.pairs) * d.B * d.Hkv;
  auto kern = dtype == kBF16 ? prefill_scores_kernel<true> : prefill_scores_kernel<false>;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kPfSmem));
  if (e != cudaSuccess) return e;
  kern<<<dim3(unsigned(grid)), kPfThreads, kPfSmem, stream>>>(kmap, a);
  return cudaGetLastError();
}

}  // namespace prism
