// Tensor-core (tcgen05) scorer for many query rows per KV head over a long shared
// context — the shared-context decode of the reference's recall (several
// questions over one cache: _dense_topk, eval_harness/attention_methods/
// reattention.py:486-498, on keys un-rotated as in _unrotate_keys :743-793 with
// undo_rotary_pos_emb, _method_base.py:336-350). Same modes and outputs as the
// mma.sync queries-as-M kernel (score_decode_wide.cu): the score matrix, the
// threshold sample (every tstride-th tile, compact columns), or the candidates at
// or above each row's threshold.
//
// The MMA: D[query row, key] over M = 128 query rows (a pair of KV heads' rows, 64
// each, held in tensor memory as the A operand, loaded once), N = 2 Tn keys (the
// tile's Tn = 128 / Hkv positions of both heads of the pair), K = 128 dimensions
// taken twice: the key un-rotated in fp32 and split into 16-bit halves hi and
// lo = round(k - hi) (bf16: hi = k truncated, |k - hi - lo| < 2^-16 |k|; fp16: hi =
// round(k)), both accumulated into the same fp32 accumulator. Of each 128 x 2 Tn
// accumulator the two diagonal blocks (a head's rows against the same head's keys)
// are kept.
//
// Roles (576 threads):
//   warp 0: idle after the set-up (the converters' first thread prefetches the
//     key tiles kAhead tiles ahead into L2 with bulk prefetches);
//   warp 1: allocates 512 TMEM columns; one lane issues the MMAs (per tile and
//     head pair: 8 k-steps on hi, 8 on lo, into the pair's 2 Tn-column accumulator;
//     two accumulator sets, so the MMAs of tile t + 1 overlap the epilogue of tile t);
//   warps 2-9: converters — thread (position, group of 8 frequency pairs): loads
//     its 16 dimensions of every head's key (L2 hits), computes the 8 angles
//     fp32(pos) * inv_freq[i] and their sin / cos once, then for every head the
//     inverse rotation r_i = x_i c + x_{i+64} s, r_{i+64} = x_{i+64} c - x_i s,
//     split into hi / lo and stored into the head's K-major, 128-byte-swizzled B
//     tiles (kBSlots slots);
//   warps 10-17: epilogue, two groups of four (one warp per TMEM lane quadrant):
//     a thread takes one 32-column chunk of its lane's (query row's) block of the
//     accumulator per tile — group g the head pair g (Hkv = 4) or the positions
//     [32 g, 32 g + 32) of the tile (Hkv = 2) — and does the mode's work. Candidates: the hit
//     mask of 32 scores (a compare each), the scores parked in shared memory when
//     there is a hit and the hits read back by index; each hit goes to this CTA's
//     segment of the row (kWideSegCap entries, no atomics; beyond it to the row's
//     list through its counter).
// Every mbarrier wait is bounded (2 s): on expiry the kernel records
// kStatusTimeout, the roles leave their loops and the TMEM is freed.
#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "rope_sincos.cuh"
#include "tc_sm100.cuh"

namespace prism {
namespace {

constexpr int kConvWarps = 8;
constexpr int kEpiWarps = 8;                  // two groups of one warp per TMEM lane quadrant
constexpr int kEpiWarp0 = 2 + kConvWarps;
constexpr int kThreads = (2 + kConvWarps + kEpiWarps) * 32;
constexpr int kBSlots = 3;
constexpr int kAhead = 8;                     // tiles prefetched into L2 ahead of the converters
// A B slot holds, per head pair, plane (hi, lo) and 64-dimension atom, the 2 Tn
// key rows of the pair (head 2 hp first) in the K-major 128-byte-swizzled layout:
// block ((hp * 2 + plane) * 2 + atom) of 2 Tn x 128 B.
constexpr uint32_t kBBytes = 65536;           // Hkv heads x (hi, lo) x Tn keys x 256 B
constexpr int kRowsPerHead = 64;              // query rows per head in the A operand
constexpr uint32_t kTmemCols = 512;           // A: Hkv/2 x 64 columns at 0; D: 2 x 128 at 256
constexpr uint32_t kDCol = 256;

constexpr uint32_t kBOff = 0;
constexpr uint32_t kParkOff = kBOff + kBSlots * kBBytes;  // 32 scores per epilogue thread
constexpr uint32_t kBarOff = kParkOff + kEpiWarps * 32 * 128;  // 32 KB
constexpr uint32_t kSmem = kBarOff + 256 + 1024;                // + alignment slack

enum TcMode : int { kTScores = 0, kTSample = 1, kTCand = 2 };

struct TcBars {
  uint64_t b_full[kBSlots], b_empty[kBSlots];
  uint64_t d_full[2], d_empty[2];
  uint64_t q_full;  // the queries are in TMEM (the four loading warps arrive)
  uint32_t tmem_base;
  int abort;
};

struct TcExtra {
  int tstride;          // kTSample: every tstride-th tile
  const float* thr;     // kTCand: per-row thresholds
  uint32_t* counts;     // kTCand: [rows, 2] (count, 0)
  uint64_t* cand;       // kTCand: [rows, cap]
  int64_t cap;
  uint64_t* seg;        // kTCand: [rows, kWideMaxSegs, kWideSegCap]
  uint32_t* segn;       // kTCand: [rows, kWideMaxSegs]
};

// Prefetch of [p, p + bytes) into L2 (bulk; 16-byte aligned, bytes a multiple of 16).
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T for one K = 16 step (A from tensor memory).
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 consecutive 32-bit columns from registers into this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
      "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
      "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// hi / lo 16-bit halves of two fp32 values (v.x in the low half of each word).
// bf16: hi truncates (the top 16 bits: one byte permute), lo = v - hi is exact in
// fp32 and rounds to bf16 — |v - hi - lo| <= 2^-9 |v - hi| < 2^-16 |v|; fp16: hi
// and lo rounded to nearest.
template <typename T>
struct SplitPair;
template <>
struct SplitPair<__nv_bfloat16> {
  __device__ __forceinline__ static void run(float2 v, uint32_t& hi, uint32_t& lo) {
    const uint32_t bx = __float_as_uint(v.x), by = __float_as_uint(v.y);
    hi = __byte_perm(bx, by, 0x7632);
    const float2 rest = __ffma2_rn(make_float2(__uint_as_float(bx & 0xffff0000u), __uint_as_float(by & 0xffff0000u)),
                                   make_float2(-1.f, -1.f), v);  // exact
    const __nv_bfloat162 l = __float22bfloat162_rn(rest);
    lo = *reinterpret_cast<const uint32_t*>(&l);
  }
};
template <>
struct SplitPair<__half> {
  __device__ __forceinline__ static void run(float2 v, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __float22half2_rn(v);
    const float2 hf = __half22float2(h);
    const __half2 l = __float22half2_rn(make_float2(v.x - hf.x, v.y - hf.y));
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
  }
};

template <typename T, bool kRope, int kMode>
__global__ void __launch_bounds__(kThreads, 1)
    wide_tc_kernel(const DecodeArgs a, const TcExtra x) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t pad = ((raw_u32 + 1023u) & ~1023u) - raw_u32;
  uint8_t* smem = smem_raw + pad;
  const uint32_t sbase = raw_u32 + pad;
  TcBars* bars = reinterpret_cast<TcBars*>(smem + kBarOff);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int Hkv = a.Hkv;
  const int Tn = 128 / Hkv;                  // positions per tile
  const int R = a.G * a.sq_n;                // query rows per KV head (<= 64)
  const int b = blockIdx.y;
  const int tstep = kMode == kTSample ? x.tstride : 1;
  const int t_begin = int(int64_t(blockIdx.x) * a.ntiles / gridDim.x);
  const int t_end = int(int64_t(blockIdx.x + 1) * a.ntiles / gridDim.x);
  const int nit = t_end - t_begin;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kBSlots; ++s) {
      mbar_init(&bars->b_full[s], kConvWarps);
      mbar_init(&bars->b_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->d_full[s], 1);
      mbar_init(&bars->d_empty[s], kEpiWarps);
    }
    mbar_init(&bars->q_full, 4);
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  asm volatile("griddepcontrol.launch_dependents;");

  // ---- the queries into TMEM (A operand): lane L of head pair hp holds query row
  // L % 64 of head 2 hp + L / 64, column c dimensions (2c, 2c + 1); the MMA issuer
  // waits for them on q_full ------------------------------------------------------
  const int quad = warp & 3;
  const int e_head = quad >> 1;                    // epilogue: head 2 hp + e_head of each pair
  const int rloc = (quad & 1) * 32 + lane;         // epilogue: row within the head (< 64)
  if (warp >= kEpiWarp0 && warp < kEpiWarp0 + 4) {  // the first group loads the queries
    const T* qg = static_cast<const T*>(a.q);
    for (int hp = 0; hp < (Hkv + 1) / 2; ++hp) {
      const int h = 2 * hp + e_head;
      const bool live = h < Hkv && rloc < R;
      const T* qr = qg + int64_t(b) * a.q_sb +
                    int64_t(h * a.G + (live ? rloc : 0) / a.sq_n) * a.q_sh +
                    int64_t(a.s0 + (live ? rloc : 0) % a.sq_n) * a.q_ss;
      // the row's bf16 (fp16) pairs are already the 32-bit columns: 16-byte loads
      // when the row is 16-byte aligned, else 4-byte ones (rows start at even
      // elements: the q strides are even)
      const bool v16 = (reinterpret_cast<uintptr_t>(qr) & 15u) == 0;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t r[32];
        if (live && v16) {
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint4 w = __ldg(reinterpret_cast<const uint4*>(qr + 64 * half) + c);
            r[4 * c] = w.x;
            r[4 * c + 1] = w.y;
            r[4 * c + 2] = w.z;
            r[4 * c + 3] = w.w;
          }
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) r[c] = live ? __ldg(reinterpret_cast<const uint32_t*>(qr + 64 * half) + c) : 0u;
        }
        tmem_st32(tmem + (uint32_t(quad * 32) << 16) + uint32_t(hp * 64 + half * 32), r);
      }
    }
    tmem_st_wait();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&bars->q_full);
  }
  // The sample pass (a few tiles per CTA) lets the converters start on the first
  // key tiles while the queries load; the long passes start every role together,
  // which measured faster for them.
  if constexpr (kMode != kTSample) __syncthreads();

  const T* kb = static_cast<const T*>(a.k) + ((a.B > 1 && a.k_sb != 0) ? int64_t(b) * a.k_sb : 0);
  auto tile_pos = [&](int it) { return (t_begin + it) * tstep * Tn; };  // first position of loop tile it

  if (warp == 0) {
    // idle
  } else if (warp == 1) {
    // ---- MMA issuer --------------------------------------------------------------
    if (lane == 0) {
      const uint32_t idesc = idesc_kind_f16(std::is_same<T, __nv_bfloat16>::value, 128, 2 * Tn);
      const uint32_t blk16 = uint32_t(2 * Tn * 128) >> 4;  // one block, in 16-byte units
      const bool q_ok = mbar_wait_bounded(&bars->q_full, 0u);
      for (int it = 0; it < nit; ++it) {
        const int bs = it % kBSlots, db = it & 1;
        bool ok = q_ok && mbar_wait_sleep_bounded(&bars->b_full[bs], uint32_t((it / kBSlots) & 1));
        if (ok && it >= 2) ok = mbar_wait_sleep_bounded(&bars->d_empty[db], uint32_t((it / 2 - 1) & 1));
        if (!ok || *reinterpret_cast<volatile int*>(&bars->abort)) {
          if (!ok) set_status(a.status, kStatusTimeout);
          bars->abort = 1;
          break;
        }
        tc_fence_after();
        // descriptor of the slot's first block; a block and a k-step are constant
        // offsets in its 16-byte address field
        const uint64_t d0 = sw128_kmajor_desc(sbase + kBOff + uint32_t(bs) * kBBytes);
        for (int hp = 0; hp < Hkv / 2; ++hp) {
          const uint32_t a_tm = tmem + uint32_t(hp * 64);
          const uint32_t d_tm = tmem + kDCol + uint32_t(db * 128 + hp * 2 * Tn);
#pragma unroll
          for (int pl = 0; pl < 2; ++pl) {
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
              const uint32_t blk = uint32_t((hp * 2 + pl) * 2 + (ks >> 2));
              tc_mma_f16_ts(d_tm, a_tm + uint32_t(ks * 8), d0 + uint64_t(blk * blk16 + uint32_t(ks & 3) * 2), idesc,
                            (pl > 0 || ks > 0) ? 1u : 0u);
            }
          }
        }
        tc_commit(&bars->b_empty[bs]);
        tc_commit(&bars->d_full[db]);
      }
    }
  } else if (warp < kEpiWarp0) {
    // ---- converters ----------------------------------------------------------------
    const int ct = (warp - 2) * 32 + lane;
    const int fg = ct & 7;  // frequency pairs [8 fg, 8 fg + 8): dimensions 8 fg.. and 64 + 8 fg..
    float inv[8];
    if (kRope) {
#pragma unroll
      for (int j = 0; j < 8; ++j) inv[j] = a.inv_freq[8 * fg + j];
    }
    const uint32_t blk = uint32_t(2 * Tn * 128);  // bytes of one (pair, plane, atom) block
    auto prefetch_tile = [&](int it) {  // every head's Tn key rows of loop tile it
      const int p0 = tile_pos(it);
      const int np = min(Tn, a.Sk - p0);
      if (np <= 0) return;
      for (int h = 0; h < Hkv; ++h) prefetch_l2(kb + int64_t(h) * a.k_sh + int64_t(p0) * 128, uint32_t(np) * 256u);
    };
    if (ct == 0)
      for (int u = 0; u < kAhead && u < nit; ++u) prefetch_tile(u);
    for (int it = 0; it < nit; ++it) {
      const int bs = it % kBSlots;
      if (ct == 0 && it + kAhead < nit) prefetch_tile(it + kAhead);
      const int p0 = tile_pos(it);
      uint8_t* bt = smem + kBOff + bs * kBBytes;
      bool waited = false, ok = true;
      for (int e = ct; e < Tn * 8; e += kConvWarps * 32) {
        const int p = e >> 3;  // position within the tile (fg is e & 7 == ct & 7)
        const int pos = p0 + p;
        // this item's 16 dimensions of every head (zeros past the end)
        uint4 wl[4], wh[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          wl[h] = make_uint4(0u, 0u, 0u, 0u);
          wh[h] = wl[h];
          if (h < Hkv && pos < a.Sk) {
            const T* row = kb + int64_t(h) * a.k_sh + int64_t(pos) * 128;
            wl[h] = __ldg(reinterpret_cast<const uint4*>(row + 8 * fg));
            wh[h] = __ldg(reinterpret_cast<const uint4*>(row + 64 + 8 * fg));
          }
        }
        float2 cs2[4], sn2[4], nsn2[4];  // (cos, sin, -sin) of frequency pairs 8 fg + 2u, +1
        if (kRope) {
          const float pf = static_cast<float>(a.pos_offset + pos);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            rope_sincos_fast(__fmul_rn(pf, inv[2 * u]), sn2[u].x, cs2[u].x);
            rope_sincos_fast(__fmul_rn(pf, inv[2 * u + 1]), sn2[u].y, cs2[u].y);
            nsn2[u] = make_float2(-sn2[u].x, -sn2[u].y);
          }
        }
        if (!waited) {  // the slot's previous tile has been read by the tensor cores
          waited = true;
          if (it >= kBSlots) ok = mbar_wait_sleep_bounded(&bars->b_empty[bs], uint32_t((it / kBSlots - 1) & 1));
          if (!__all_sync(0xffffffffu, ok) || *reinterpret_cast<volatile int*>(&bars->abort)) {
            ok = false;
            break;
          }
        }
        const uint32_t sw = uint32_t(((fg ^ (p & 7)) * 16));  // the chunk's swizzled slot in the row
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          if (h >= Hkv) break;
          const uint32_t wlo[4] = {wl[h].x, wl[h].y, wl[h].z, wl[h].w};
          const uint32_t whi[4] = {wh[h].x, wh[h].y, wh[h].z, wh[h].w};
          uint32_t hl[4], ll[4], hh[4], lh[4];  // hi / lo of dimensions 8 fg.. and 64 + 8 fg..
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            float2 xv, yv;  // x: dims 8 fg + 2u, +1; y: the same + 64
            Unpack<T>::run(wlo[u], xv.x, xv.y);
            Unpack<T>::run(whi[u], yv.x, yv.y);
            float2 r = xv, q = yv;
            if (kRope) {  // packed fp32x2: r = x c + y s, q = y c - x s
              r = __ffma2_rn(xv, cs2[u], __fmul2_rn(yv, sn2[u]));
              q = __ffma2_rn(yv, cs2[u], __fmul2_rn(xv, nsn2[u]));
            }
            SplitPair<T>::run(r, hl[u], ll[u]);
            SplitPair<T>::run(q, hh[u], lh[u]);
          }
          // row (h & 1) Tn + p of the pair's blocks: hi atom 0, hi atom 1, lo atom 0, lo atom 1
          uint8_t* hip = bt + uint32_t((h >> 1) * 4) * blk + uint32_t((h & 1) * Tn + p) * 128 + sw;
          *reinterpret_cast<uint4*>(hip) = make_uint4(hl[0], hl[1], hl[2], hl[3]);
          *reinterpret_cast<uint4*>(hip + blk) = make_uint4(hh[0], hh[1], hh[2], hh[3]);
          *reinterpret_cast<uint4*>(hip + 2 * blk) = make_uint4(ll[0], ll[1], ll[2], ll[3]);
          *reinterpret_cast<uint4*>(hip + 3 * blk) = make_uint4(lh[0], lh[1], lh[2], lh[3]);
        }
      }
      if (!ok) {
        set_status(a.status, kStatusTimeout);
        bars->abort = 1;
        break;
      }
      fence_proxy_async_smem();  // the B tiles are read by the tensor cores
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->b_full[bs]);
    }
  } else {
    // ---- epilogue: thread = query row rloc of head 2 hp + e_head, chunk g ------------
    // a dependent launch: the thresholds (and the buffers the kernel before may still
    // read) are settled after the wait; the other roles read only the keys
    grid_dependency_wait();
    const int g = (warp - kEpiWarp0) >> 2;         // epilogue group
    const int hp = Hkv == 4 ? g : 0;               // the head pair of this thread's row
    const int h = 2 * hp + e_head;
    const bool live = rloc < R;
    const int rr = live ? rloc : 0;
    const int s_abs = a.s0 + rr % a.sq_n;
    const int64_t srow = (int64_t(b) * a.Hq + int64_t(h) * a.G + rr / a.sq_n) * a.Sq + s_abs;
    const int64_t vis = a.causal ? a.causal_offset + s_abs : INT64_MAX;
    const int64_t rend = a.causal ? min(int64_t(a.Sk), a.causal_offset + s_abs + 1) : int64_t(a.Sk);
    const float thr = kMode == kTCand && live ? x.thr[srow] : 0.f;
    // accumulator column of this chunk and its first position / sample column in the tile
    const uint32_t col = Hkv == 4 ? uint32_t(hp * 2 * Tn + e_head * Tn) : uint32_t(e_head * Tn + 32 * g);
    const int off = Hkv == 4 ? 0 : 32 * g;
    uint32_t nst = 0;  // candidates of the row found by this thread
    const int64_t sbase_ = (srow * kWideMaxSegs + 2 * blockIdx.x + g) * kWideSegCap;
    const int et = (warp - kEpiWarp0) * 32 + lane;
    uint8_t* park = smem + kParkOff + uint32_t(et) * 16;  // chunk q at + q * 256 * 16
    const uint32_t dlane = tmem + (uint32_t(quad * 32) << 16) + kDCol + col;
    for (int it = 0; it < nit; ++it) {
      const int db = it & 1;
      if (!__all_sync(0xffffffffu, mbar_wait_sleep_bounded(&bars->d_full[db], uint32_t((it >> 1) & 1)))) {
        set_status(a.status, kStatusTimeout);
        bars->abort = 1;
        break;
      }
      tc_fence_after();
      uint32_t vv[32];
      tmem_ld32(dlane + uint32_t(db * 128), vv);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->d_empty[db]);
      if (!live) continue;
      const int pb = tile_pos(it) + off;
      if (kMode == kTCand) {
        const int64_t lim = rend - pb;
        uint32_t m = 0;
#pragma unroll
        for (int j = 0; j < 32; ++j) m |= (__uint_as_float(vv[j]) < thr ? 0u : 1u) << j;  // NaN: a hit
        m &= lim >= 32 ? 0xffffffffu : (lim <= 0 ? 0u : ((1u << lim) - 1u));
        if (m != 0u) {
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<uint4*>(park + q * kEpiWarps * 32 * 16) =
                make_uint4(vv[4 * q], vv[4 * q + 1], vv[4 * q + 2], vv[4 * q + 3]);
          while (m) {
            const int j = __ffs(m) - 1;
            m &= m - 1;
            const uint32_t bits = *reinterpret_cast<const uint32_t*>(park + (j >> 2) * kEpiWarps * 32 * 16 + (j & 3) * 4);
            const uint64_t pk = (uint64_t(bits) << 32) | uint64_t(~uint32_t(pb + j));
            if (nst < uint32_t(kWideSegCap)) {
              x.seg[sbase_ + nst] = pk;
            } else {  // the segment is full: the row's list, through its counter
              const uint32_t slot = atomicAdd(&x.counts[2 * srow], 1u);
              if (slot < uint64_t(x.cap)) x.cand[srow * x.cap + slot] = pk;
            }
            ++nst;
          }
        }
      } else {
        const int cb = (t_begin + it) * Tn + off;  // kTSample: the chunk's first sample column
        float* o = a.scores + srow * a.ld + (kMode == kTSample ? cb : pb);
        const int64_t lim = kMode == kTSample ? INT64_MAX : a.Sk - pb;  // sample: every column
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          float w[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int64_t pos = pb + j + u;
            w[u] = pos < a.Sk && pos <= vis ? __uint_as_float(vv[j + u]) : -INFINITY;
          }
          if (j + 4 <= lim) {
            *reinterpret_cast<float4*>(o + j) = make_float4(w[0], w[1], w[2], w[3]);
          } else {
#pragma unroll
            for (int u = 0; u < 4; ++u)
              if (j + u < lim) o[j + u] = w[u];
          }
        }
      }
    }
    if (kMode == kTCand && live)
      x.segn[srow * kWideMaxSegs + 2 * blockIdx.x + g] = min(nst, uint32_t(kWideSegCap));
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <typename T, bool kRope, int kMode>
cudaError_t launch_tc(const DecodeArgs& a, int num_sms, const TcExtra& x, cudaStream_t stream) {
  auto kern = wide_tc_kernel<T, kRope, kMode>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmem));
  if (e != cudaSuccess) return e;
  const int Tn = 128 / a.Hkv;
  DecodeArgs d = a;
  d.ntiles = (a.Sk + Tn - 1) / Tn;
  if (kMode == kTSample) d.ntiles = (d.ntiles + x.tstride - 1) / x.tstride;  // sampled tiles
  int ctas = num_sms;
  if (a.B > 1) ctas = (num_sms + a.B - 1) / a.B;
  ctas = max(1, min(ctas, d.ntiles));
  return launch_maybe_dependent(kern, dim3(ctas, a.B), dim3(kThreads), kSmem, true, stream, d, x);
}

template <int kMode>
cudaError_t launch_tc_mode(const DecodeArgs& a, int dtype, int num_sms, const TcExtra& x, cudaStream_t stream) {
  const bool rope = a.inv_freq != nullptr;
  if (dtype == kBF16)
    return rope ? launch_tc<__nv_bfloat16, true, kMode>(a, num_sms, x, stream)
                : launch_tc<__nv_bfloat16, false, kMode>(a, num_sms, x, stream);
  return rope ? launch_tc<__half, true, kMode>(a, num_sms, x, stream)
              : launch_tc<__half, false, kMode>(a, num_sms, x, stream);
}

}  // namespace

bool wide_tc_supported(const DecodeArgs& a) {
  const int H = a.Hkv;
  const bool q_ok = (reinterpret_cast<uintptr_t>(a.q) & 3u) == 0 && a.q_sb % 2 == 0 && a.q_sh % 2 == 0 &&
                    a.q_ss % 2 == 0;  // 4-byte query words
  return q_ok && (H == 2 || H == 4) && a.G * a.sq_n <= kRowsPerHead && a.G * a.sq_n >= 1 &&
         (reinterpret_cast<uintptr_t>(a.scores) & 15u) == 0 && a.ld % 4 == 0;
}

cudaError_t launch_wide_tc_scores(const DecodeArgs& a, int dtype, int num_sms, cudaStream_t stream) {
  return launch_tc_mode<kTScores>(a, dtype, num_sms, TcExtra{1, nullptr, nullptr, nullptr, 0, nullptr, nullptr},
                                  stream);
}

cudaError_t launch_wide_tc_sample(const DecodeArgs& a, int dtype, int num_sms, cudaStream_t stream) {
  return launch_tc_mode<kTSample>(
      a, dtype, num_sms, TcExtra{kWideSampleStride, nullptr, nullptr, nullptr, 0, nullptr, nullptr}, stream);
}

cudaError_t launch_wide_tc_candidates(const DecodeArgs& a, int dtype, const float* thr, uint32_t* counts,
                                      uint64_t* cand, int64_t cap, uint64_t* seg, uint32_t* segn,
                                      int num_sms, cudaStream_t stream) {
  if (2 * num_sms > kWideMaxSegs) return cudaErrorInvalidValue;
  return launch_tc_mode<kTCand>(a, dtype, num_sms, TcExtra{1, thr, counts, cand, cap, seg, segn}, stream);
}

}  // namespace prism
