// Decode scorer on register tensor-core tiles shared by head pairs (bf16 keys,
// Hkv in {2, 4, 8}, at most 4 query rows per KV head) — the 128K / 1M decode
// shapes of the reference's recall (reattention.py:486-498 with q_len = 1,
// keys un-rotated as in _unrotate_keys, reattention.py:743-793).
//
// One mma.sync m16n8k8 TF32 tile covers 8 key positions x 2 KV heads:
//   A rows 0..7  = positions p..p+7 of head h0, rows 8..15 = the same positions
//   of head h1 (rotated keys, 8 dims per k-step);
//   B columns 0..3 = the (<= 4) query rows of h0, columns 4..7 those of h1.
// Lane (g, c) owns A rows g and g+8 — the SAME position in two heads — and
// rotation pairs [16c, 16c+16) of both halves, so the RoPE cos/sin of its 16
// pairs (computed once per 8-position sub-tile, 16 angles per lane) stay in
// registers for every head pair: no shared cos/sin table, no block barrier.
// Of the tile's outputs, lanes c < 2 keep rows (h0 key, h0 queries) and lanes
// c >= 2 keep (h1 key, h1 queries); the off-diagonal quarters are discarded.
//
// Precision: the tensor core reads a TF32 operand's top 19 bits and ignores the
// rest, i.e. it truncates. The cos/sin factors are therefore scaled by
// (1 + 2^-11), so that the rotated key enters the MMA as trunc(k_raw * (1 + 2^-11)):
// for k_raw = m * 2^e (1 <= m < 2) the scale adds m/2 TF32 ulps before the
// truncation, and the result lies within (-(1 - m/2), m/2] ulps of k_raw, a
// relative error below 2^-11 — the bound of round-to-nearest, at no per-element
// cost. bf16 queries (and un-rotated bf16 keys) are exact in TF32; accumulation
// is fp32. The score error is at most 2^-11 * sum_i |q_i k_i| <= 0.49 of the
// 1e-3 * ||q|| ||k|| tolerance.
//
// Memory: each warp streams its own copies (16 positions x one head pair, one
// tiled TMA copy of 8 KB with 4 KB contiguous per head) through a private 3-stage
// ring, two copies in flight per warp; 8 warps (two per scheduler) hide each
// other's latencies. The query fragments live in a shared table, so registers
// hold only keys, angles and accumulators.
#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "rope_sincos.cuh"
#include "tensor_map.h"

namespace prism {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kStages = 3;
constexpr int kP = 8;              // positions per sub-tile (MMA rows per head)
constexpr int kSubs = 2;           // sub-tiles per copy
constexpr int kPc = kP * kSubs;    // positions per copy: 4 KB contiguous per head
constexpr int kMaxPairs = 4;       // Hkv <= 8
constexpr int kPairsPerCopy = 1;   // one TMA copy holds one head pair (2 heads)
constexpr float kTruncScale = 1.0f + 0x1.0p-11f;  // see the precision note

struct __align__(16) HpTail {
  // B fragments in fragment order: bfrag[hp][ks][lane] = (b0, b1) of the k-step ks
  // MMA of head pair hp, as fp32 (bf16 queries are exact in TF32)
  float2 bfrag[kMaxPairs][16][32];
  uint64_t full[kWarps][kStages];
  int slice_of[kWarps][4];  // the warp's q-th slice (q mod 4), written by its lane 0 at the claim
  unsigned int next;         // next unclaimed slice of this CTA's range
};

__device__ __forceinline__ void mma_tf32(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <bool kRope, bool kDyn>
__global__ void __launch_bounds__(kThreads, 1)
    decode_hp_kernel(const __grid_constant__ CUtensorMap kmap, const DecodeArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int Hkv = a.Hkv;
  const int npairs = Hkv / 2;
  const int ppc = npairs < kPairsPerCopy ? npairs : kPairsPerCopy;  // pairs per copy
  const int copies = npairs / ppc;                                  // copies per sub-tile: 1, 2, 4
  const int cshift = copies == 4 ? 2 : (copies == 2 ? 1 : 0);
  const int R = a.G * a.sq_n;  // <= 4
  const uint32_t copy_bytes = uint32_t(ppc) * 2 * kPc * kRowBytes;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2;  // position g of the sub-tile; B column g
  const int c = lane & 3;   // rotation pairs [16c, 16c+16)
  const int b = blockIdx.y;
  HpTail* tail = reinterpret_cast<HpTail*>(smem + kWarps * kStages * copy_bytes);
  uint8_t* ring = smem + warp * kStages * copy_bytes;
  uint64_t* full = tail->full[warp];

  // Work: slices of kPc positions (all KV heads). Static (kDyn false): each warp
  // streams a fixed contiguous range. Dynamic (long rows, many slices per warp):
  // two levels, so that warps and SMs that stream faster take more slices and all
  // finish together — the first 7/8 of the slices are split into one contiguous
  // range per CTA, whose warps take them one at a time from a shared-memory
  // counter (a warp's first slice is fixed: the range start plus its warp
  // number); the last 1/8 is a pool that CTAs done with their range claim from a
  // global counter per batch row (a.work, zero at launch). A slice is claimed
  // when lane 0 issues its first copy.
  const int nsub = (a.Sk + kPc - 1) / kPc;
  const int64_t gw = int64_t(blockIdx.x) * kWarps + warp, nw = int64_t(gridDim.x) * kWarps;
  const int i_begin = int(gw * nsub / nw), i_end = int((gw + 1) * nsub / nw);
  const int ncopies = (i_end - i_begin) * copies;
  unsigned int* const work = kDyn ? a.work + blockIdx.y : nullptr;
  const int nstat = nsub - nsub / 8;
  const int cta_begin = int(int64_t(blockIdx.x) * nstat / gridDim.x);
  const int cta_end = int(int64_t(blockIdx.x + 1) * nstat / gridDim.x);
  int* const slice_of = tail->slice_of[warp];
  bool first = true;       // lane 0: the warp's first claim
  bool exhausted = false;  // lane 0: no slice left to issue
  auto claim = [&]() -> int {
    if (first) {
      first = false;
      if (cta_begin + warp < cta_end) return cta_begin + warp;
    }
    const int v = int(atomicAdd(&tail->next, 1u));
    if (v < cta_end) return v;
    const int w = nstat + int(atomicAdd(work, 1u));
    return w < nsub ? w : nsub;
  };
  if (kDyn) {
    if (tid == 0) tail->next = unsigned(cta_begin + kWarps);
    __syncthreads();
  }

  asm volatile("griddepcontrol.launch_dependents;");
  if (lane == 0) {
    if (warp == 0) asm volatile("prefetch.tensormap [%0];" ::"l"(&kmap) : "memory");
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncwarp();

  const int kb_coord = (a.B > 1 && a.k_sb != 0) ? b : 0;
  // copy t of this warp (lane 0): part t % copies (heads [part * 2ppc, +2ppc)) of
  // the warp's (t / copies)-th slice, claimed with its first part
  auto issue = [&](int t, int s) {
    const int q = t >> cshift;
    const int part = t & (copies - 1);
    int i;
    if (!kDyn) {
      if (t >= ncopies) return;
      i = i_begin + q;
    } else {
      if (exhausted) return;
      if (part == 0) {
        i = claim();
        slice_of[q & 3] = i;
        if (i >= nsub) {
          exhausted = true;
          return;
        }
      } else {
        i = slice_of[q & 3];
      }
    }
    const uint64_t pol = l2_policy_evict_first();
    mbar_arrive_expect_tx(&full[s], copy_bytes);
    tma_load_4d(ring + s * copy_bytes, &kmap, 0, i * kPc, part * 2 * ppc, kb_coord, &full[s], pol);
  };
  if (lane == 0) {
    for (int t = 0; t < kStages; ++t) issue(t, t);
  }
  __syncwarp();

  // ---- per-lane constants ------------------------------------------------------------
  // this lane's 16 frequencies (pairs 16c + 2i, 16c + 2i + 1)
  float2 inv[8];
  if (kRope) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      inv[i] = make_float2(a.inv_freq[16 * c + 2 * i], a.inv_freq[16 * c + 2 * i + 1]);
  }
  // B fragments: lane (g, c) of k-step ks holds rows k = c and c + 4 of column g,
  // i.e. q[row][d] and q[row][d + 1] with row = B column g (h0 row g for g < 4, h1
  // row g - 4 otherwise) and d = 16c + 2ks (ks < 8) or 64 + 16c + 2(ks - 8)
  {
    const __nv_bfloat16* qg = static_cast<const __nv_bfloat16*>(a.q);
    for (int e = tid; e < kMaxPairs * 16 * 32; e += kThreads) {
      const int ln = e & 31, ks = (e >> 5) & 15, hp = e >> 9;
      const int gg = ln >> 2, cc4 = ln & 3;
      const int qrow = gg & 3, h = 2 * hp + (gg >> 2);
      float2 v = make_float2(0.f, 0.f);
      if (hp < npairs && qrow < R) {
        const __nv_bfloat16* qr = qg + int64_t(b) * a.q_sb + int64_t(h * a.G + qrow / a.sq_n) * a.q_sh +
                                  int64_t(a.s0 + qrow % a.sq_n) * a.q_ss;
        const int d = ks < 8 ? 16 * cc4 + 2 * ks : 64 + 16 * cc4 + 2 * (ks - 8);
        v = make_float2(__bfloat162float(qr[d]), __bfloat162float(qr[d + 1]));
      }
      tail->bfrag[hp][ks][ln] = v;
    }
  }
  __syncthreads();
  const uint32_t bfrag_lane = smem_u32(&tail->bfrag[0][0][lane]);
  // outputs of this lane: head h0 (c < 2) or h1 (c >= 2) of each pair, query
  // rows r0 = (2c) & 3 and r0 + 1
  const int r0 = (2 * c) & 3;
  const bool wr0 = r0 < R, wr1 = r0 + 1 < R;
  const int s_abs0 = a.s0 + r0 % a.sq_n, s_abs1 = a.s0 + (r0 + 1) % a.sq_n;
  const int64_t vis0 = a.causal ? a.causal_offset + s_abs0 : INT64_MAX;
  const int64_t vis1 = a.causal ? a.causal_offset + s_abs1 : INT64_MAX;
  const int hsel = c >> 1;
  // score row of (head 2hp + hsel, query row r0) = row_base + hp * pair_stride;
  // query row r0 + 1 adds row1_delta
  const int64_t row_base =
      ((int64_t(b) * a.Hq + hsel * a.G + r0 / a.sq_n) * a.Sq + s_abs0) * a.ld;
  const int64_t row1_delta =
      ((int64_t((r0 + 1) / a.sq_n) - r0 / a.sq_n) * a.Sq + (s_abs1 - s_abs0)) * a.ld;
  const int64_t pair_stride = int64_t(2) * a.G * a.Sq * a.ld;
  const uint32_t ring_u32 = smem_u32(ring);
  const uint32_t lane_off = uint32_t(g) * kRowBytes + 32 * c;

  int t = 0;  // copies consumed
  for (int qs = 0;; ++qs) {
    // dynamic: the slice lane 0 claimed (written before an earlier __syncwarp)
    const int i = kDyn ? slice_of[qs & 3] : i_begin + qs;
    if (kDyn ? i >= nsub : i >= i_end) break;
    // cos/sin of this lane's 16 pairs at its position in each sub-tile (overlaps
    // the copy), pre-scaled for the truncating TF32 operand
    // (each value twice: the packed FMAs below pair the two heads of a head
    // pair, which share the angle)
    float2 cc[kSubs][16], ss[kSubs][16];
    if (kRope) {
#pragma unroll
      for (int sb = 0; sb < kSubs; ++sb) {
        const float pf = static_cast<float>(a.pos_offset + i * kPc + sb * kP + g);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            float sv, cv;
            rope_sincos_fast(__fmul_rn(pf, e ? inv[q].y : inv[q].x), sv, cv);
            sv *= kTruncScale;
            cv *= kTruncScale;
            ss[sb][2 * q + e] = make_float2(sv, sv);
            cc[sb][2 * q + e] = make_float2(cv, cv);
          }
        }
      }
    }
    uint32_t st = 0;
#pragma unroll
    for (int hp = 0; hp < kMaxPairs; ++hp) {
      if (hp >= npairs) break;
      const int slot = hp & (ppc - 1);  // pair within the current copy
      if (slot == 0) {
        if (hp > 0) {  // release the previous copy of this block
          __syncwarp();
          if (lane == 0) issue(t - 1 + kStages, (t - 1) % kStages);
        }
        const int s = t % kStages;
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full[s], (t / kStages) & 1))) {
          set_status(a.status, kStatusTimeout);
          return;
        }
        st = ring_u32 + s * copy_bytes + lane_off;
        ++t;
      }
#pragma unroll
      for (int sb = 0; sb < kSubs; ++sb) {
        const int pos = i * kPc + sb * kP + g;
        // A rows: g -> head 2hp, g+8 -> head 2hp+1 (same position); packed bf16
        // words: [row][0..7] dims 16c..16c+15, [row][8..15] dims 64+16c..
        uint32_t kw[2][16];
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          const uint32_t row = st + uint32_t((2 * slot + rr) * kPc + sb * kP) * kRowBytes;
          const uint4 w0 = lds128_u32(row), w1 = lds128_u32(row + 16);
          const uint4 w2 = lds128_u32(row + 128), w3 = lds128_u32(row + 144);
          kw[rr][0] = w0.x; kw[rr][1] = w0.y; kw[rr][2] = w0.z; kw[rr][3] = w0.w;
          kw[rr][4] = w1.x; kw[rr][5] = w1.y; kw[rr][6] = w1.z; kw[rr][7] = w1.w;
          kw[rr][8] = w2.x; kw[rr][9] = w2.y; kw[rr][10] = w2.z; kw[rr][11] = w2.w;
          kw[rr][12] = w3.x; kw[rr][13] = w3.y; kw[rr][14] = w3.z; kw[rr][15] = w3.w;
        }
        // pair q (dims 16c+2q, +1 and +64) feeds k-step q (lo half, acc0) and
        // k-step 8+q (hi half, acc1). Packed operands pair the two heads:
        // x = head 2hp (A row g), y = head 2hp+1 (A row g+8), so that the
        // rotated values land in the MMA's A registers in order
        // (row g, row g+8) for dims 16c+2q and 16c+2q+1.
        float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const uint32_t w0 = kw[0][q], w1 = kw[1][q], u0 = kw[0][8 + q], u1 = kw[1][8 + q];
          const float2 L0 = make_float2(__uint_as_float(w0 << 16), __uint_as_float(w1 << 16));
          const float2 L1 = make_float2(__uint_as_float(w0 & 0xffff0000u), __uint_as_float(w1 & 0xffff0000u));
          const float2 H0 = make_float2(__uint_as_float(u0 << 16), __uint_as_float(u1 << 16));
          const float2 H1 = make_float2(__uint_as_float(u0 & 0xffff0000u), __uint_as_float(u1 & 0xffff0000u));
          float2 klo0, klo1, khi0, khi1;
          if (kRope) {
            const float2 s0 = ss[sb][2 * q], s1 = ss[sb][2 * q + 1];
            const float2 c0 = cc[sb][2 * q], c1 = cc[sb][2 * q + 1];
            klo0 = __ffma2_rn(H0, s0, __fmul2_rn(L0, c0));
            klo1 = __ffma2_rn(H1, s1, __fmul2_rn(L1, c1));
            khi0 = __ffma2_rn(L0, make_float2(-s0.x, -s0.y), __fmul2_rn(H0, c0));
            khi1 = __ffma2_rn(L1, make_float2(-s1.x, -s1.y), __fmul2_rn(H1, c1));
          } else {
            klo0 = L0;
            klo1 = L1;
            khi0 = H0;
            khi1 = H1;
          }
          const uint2 bl = lds64_u32(bfrag_lane + uint32_t((hp * 16 + q) * 32 * 8));
          const uint2 bh = lds64_u32(bfrag_lane + uint32_t((hp * 16 + 8 + q) * 32 * 8));
          mma_tf32(acc0, __float_as_uint(klo0.x), __float_as_uint(klo0.y), __float_as_uint(klo1.x),
                   __float_as_uint(klo1.y), bl.x, bl.y);
          mma_tf32(acc1, __float_as_uint(khi0.x), __float_as_uint(khi0.y), __float_as_uint(khi1.x),
                   __float_as_uint(khi1.y), bh.x, bh.y);
        }
        // d0,d1: (h0 key, columns 2c, 2c+1); d2,d3: (h1 key, same columns)
        const float v0 = hsel ? acc0[2] + acc1[2] : acc0[0] + acc1[0];
        const float v1 = hsel ? acc0[3] + acc1[3] : acc0[1] + acc1[1];
        if (pos < a.Sk) {
          const int64_t ro = row_base + int64_t(hp) * pair_stride;
          const float s0 = int64_t(pos) > vis0 ? -INFINITY : v0;
          const float s1 = int64_t(pos) > vis1 ? -INFINITY : v1;
          if (wr0) a.scores[ro + pos] = s0;
          if (wr1) a.scores[ro + row1_delta + pos] = s1;
        }
      }
    }
    __syncwarp();  // every lane is done with the last copy of this block
    if (lane == 0) issue(t - 1 + kStages, (t - 1) % kStages);
    if (kDyn) __syncwarp();  // the claims lane 0 just made are visible to the warp
  }
}

size_t hp_smem_bytes(int Hkv) {
  const int heads_per_copy = Hkv < 2 * kPairsPerCopy ? Hkv : 2 * kPairsPerCopy;
  return size_t(kWarps) * kStages * heads_per_copy * kPc * kRowBytes + sizeof(HpTail);
}

template <bool kRope>
cudaError_t launch_hp(const DecodeArgs& a, int num_sms, cudaStream_t stream) {
  const size_t smem = hp_smem_bytes(a.Hkv);
  const int nsub_ = (a.Sk + kPc - 1) / kPc;
  const int ctas_ = a.B > 1 ? (num_sms + a.B - 1) / a.B : num_sms;
  // dynamic distribution once each warp has many slices (long rows): its claims
  // cost less than the imbalance they remove
  const bool dyn = a.work != nullptr && nsub_ >= 16 * ctas_ * kWarps;
  auto kern = dyn ? decode_hp_kernel<kRope, true> : decode_hp_kernel<kRope, false>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  CUtensorMap kmap;
  const int heads_per_copy = a.Hkv < 2 * kPairsPerCopy ? a.Hkv : 2 * kPairsPerCopy;
  e = make_key_tensor_map(&kmap, a.k, kBF16, a.B, a.Hkv, a.Sk, a.k_sb, a.k_sh, kPc, heads_per_copy);
  if (e != cudaSuccess) return e;
  const int nsub = (a.Sk + kPc - 1) / kPc;
  int ctas = num_sms;
  if (a.B > 1) ctas = (num_sms + a.B - 1) / a.B;
  ctas = max(1, min(ctas, (nsub + kWarps - 1) / kWarps));
  kern<<<dim3(ctas, a.B), kThreads, smem, stream>>>(kmap, a);
  return cudaGetLastError();
}

}  // namespace

bool decode_hp_supported(const DecodeArgs& a, int dtype) {
  const int R = a.G * a.sq_n;
  const int H = a.Hkv;
  const bool q_ok = (reinterpret_cast<uintptr_t>(a.q) & 3u) == 0 && a.q_sb % 2 == 0 &&
                    a.q_sh % 2 == 0 && a.q_ss % 2 == 0;
  return dtype == kBF16 && R <= 4 && (H == 2 || H == 4 || H == 8) && q_ok;
}

cudaError_t launch_decode_scores_hp(const DecodeArgs& a, int num_sms, cudaStream_t stream) {
  return a.inv_freq != nullptr ? launch_hp<true>(a, num_sms, stream)
                               : launch_hp<false>(a, num_sms, stream);
}

}  // namespace prism
