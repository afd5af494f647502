// Decode scorer, fast path for at most 4 query rows per KV head (GQA decode:
// Hq/Hkv <= 4 query heads per KV head at one query position) — the decode
// shape of the reference's recall (reattention.py:486-498 with q_len = 1) —
// and Hkv in {1, 2, 4, 8, 16}.
//
// Same math as score_decode.cu (inverse RoPE fused into the key load, fp32
// dot products), organised for instruction issue and shared-memory bandwidth:
//
//  * a stage holds Tp key positions of EVERY KV head of one batch row, brought
//    in by ONE tiled TMA copy (a 4-D tensor map over [B, Hkv, Sk, 128], box
//    {128, Tp, Hkv, 1}; rows past Sk are zero-filled), 32 KB per stage; four
//    stages, three tiles in flight while one is consumed;
//  * per tile, all threads compute the RoPE cos/sin of Tp positions x 64
//    frequencies into a double-buffered shared table; thread 0 then issues the
//    copies of tile t+3 and alone waits for tile t's bytes, and the block
//    barrier that follows publishes both (no thread spins on the mbarrier; the
//    barrier also proves tile t-1's stage and table are no longer read);
//  * 16 warps, 32 work items (kv head, 4 positions) per tile, 2 per warp, both
//    of the same head: each warp keeps its head's query rows in registers
//    (4 rows x 16 values per lane) for the whole kernel, and every address of
//    an item is precomputed once;
//  * 8 lanes per key, each owning rotation pairs [8j, 8j+8) of the two halves.
//    Key rows are read conflict-free as laid out; the cos/sin table gives lane
//    j a contiguous 64-byte block at 80*j bytes (rows padded to 640 B), so the
//    8 lanes of a key hit 8 distinct bank groups with immediate offsets;
//  * rotation and dot products in packed fp32x2 FMA (__ffma2_rn / __fmul2_rn).
#include "common.cuh"
#include "kernels.h"
#include "rope_sincos.cuh"
#include "tensor_map.h"

#include <type_traits>

namespace prism {
namespace {

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kStages = 4;
constexpr int kMaxR = 4;
constexpr int kItemsPerWarp = 2;
constexpr int kCsRow = 640;  // bytes per position in the cos/sin table (512 + padding)

struct __align__(16) G4Tail {
  uint64_t full[kStages];
  float inv_freq[64];
  int abort;
};

// physical 16-byte chunk of logical chunk qc (pairs 2qc, 2qc+1): lane j = qc/4
// owns chunks 5j .. 5j+3
__device__ __forceinline__ int cs_phys(int qc) { return 5 * (qc >> 2) + (qc & 3); }

template <typename T>
__device__ __forceinline__ void unpack4(const uint4& v, float2 out[4]) {
  Unpack<T>::run(v.x, out[0].x, out[0].y);
  Unpack<T>::run(v.y, out[1].x, out[1].y);
  Unpack<T>::run(v.z, out[2].x, out[2].y);
  Unpack<T>::run(v.w, out[3].x, out[3].y);
}

template <typename T, bool kRope>
__global__ void __launch_bounds__(kThreads, 1)
    decode_g4_kernel(const __grid_constant__ CUtensorMap kmap, const DecodeArgs a, int Tp) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int Hkv = a.Hkv;
  const int R = a.G * a.sq_n;  // <= 4
  const uint32_t stage_bytes = uint32_t(Hkv) * Tp * kRowBytes;
  uint8_t* stages = smem;
  uint8_t* cs_tab = smem + kStages * stage_bytes;  // [2][Tp][kCsRow]
  G4Tail* tail = reinterpret_cast<G4Tail*>(cs_tab + 2 * Tp * kCsRow);

  const int tid = threadIdx.x;
  const int b = blockIdx.y;
  const int t_begin = static_cast<int>(int64_t(blockIdx.x) * a.ntiles / gridDim.x);
  const int t_end = static_cast<int>(int64_t(blockIdx.x + 1) * a.ntiles / gridDim.x);

  // let the selection kernel (launched with programmatic stream serialization)
  // be scheduled while this grid drains; it waits for our completion itself
  asm volatile("griddepcontrol.launch_dependents;");
  if (tid == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(&kmap) : "memory");
    for (int s = 0; s < kStages; ++s) mbar_init(&tail->full[s], 1);
    tail->abort = 0;
    fence_mbar_init();
  }
  if (kRope) {
    for (int i = tid; i < kHeadDim / 2; i += kThreads) tail->inv_freq[i] = a.inv_freq[i];
  }

  // ---- per-lane constants ------------------------------------------------------------
  const int warp = tid >> 5, lane = tid & 31;
  const int j = lane & 7;    // rotation pairs [8j, 8j+8)
  const int pl = lane >> 3;  // key within an item (0..3)
  const int npass = Tp / 4;
  const int nitems = Hkv * npass;   // 16 or 32
  const int ipw = nitems / kWarps;  // 1 or 2 items per warp
  const int item0 = warp * ipw;
  const int h = item0 / npass;  // kv head of this warp's items
  int k_off[kItemsPerWarp], cs_off[kItemsPerWarp], p_of[kItemsPerWarp];
#pragma unroll
  for (int i = 0; i < kItemsPerWarp; ++i) {
    const int p = 4 * ((item0 % npass) + i) + pl;  // key position within the tile
    p_of[i] = p;
    k_off[i] = (h * Tp + p) * kRowBytes + 16 * j;
    cs_off[i] = p * kCsRow + 80 * j;
  }
  // query rows of head h: row r -> (q head h*G + r / sq_n, query s0 + r % sq_n)
  float2 q_lo[kMaxR][4], q_hi[kMaxR][4];  // dims 8j+2m, 8j+2m+1 (and +64)
  {
    const T* qg = static_cast<const T*>(a.q);
#pragma unroll
    for (int r = 0; r < kMaxR; ++r) {
      const int rr = min(r, R - 1);
      const T* qr = qg + int64_t(b) * a.q_sb + int64_t(h * a.G + rr / a.sq_n) * a.q_sh +
                    int64_t(a.s0 + rr % a.sq_n) * a.q_ss;
      const uint4 lo = *reinterpret_cast<const uint4*>(qr + 8 * j);
      const uint4 hi = *reinterpret_cast<const uint4*>(qr + 64 + 8 * j);
      unpack4<T>(lo, q_lo[r]);
      unpack4<T>(hi, q_hi[r]);
    }
  }
  // output row of this lane: row r = j/2 of the head's group
  const int r_lane = j >> 1;
  const bool writer = (j & 1) == 0 && r_lane < R;
  const int s_abs = a.s0 + r_lane % a.sq_n;
  float* const out =
      a.scores + ((int64_t(b) * a.Hq + h * a.G + r_lane / a.sq_n) * a.Sq + s_abs) * a.ld;
  const int64_t vis_limit = a.causal ? a.causal_offset + s_abs : INT64_MAX;
  __syncthreads();

  const int kb_coord = (a.B > 1 && a.k_sb != 0) ? b : 0;
  // one tensor copy brings tile t (all KV heads) into stage s (thread 0 only)
  auto issue = [&](int t, int s) {
    const uint64_t pol = l2_policy_evict_first();
    mbar_arrive_expect_tx(&tail->full[s], stage_bytes);
    tma_load_4d(stages + s * stage_bytes, &kmap, 0, t * Tp, 0, kb_coord, &tail->full[s], pol);
  };
  if (tid == 0) {
    for (int k = 0; k < kStages - 1 && t_begin + k < t_end; ++k) issue(t_begin + k, k);
  }

  int it = 0;
  for (int t = t_begin; t < t_end; ++t, ++it) {
    const int p0 = t * Tp;
    uint8_t* cs_buf = cs_tab + (it & 1) * Tp * kCsRow;
    if (kRope) {
      for (int idx = tid; idx < Tp * 32; idx += kThreads) {
        const int p = idx >> 5, qc = idx & 31;
        const float pf = static_cast<float>(a.pos_offset + p0 + p);
        float4 v;  // (cos f0, cos f1, sin f0, sin f1) of freqs 2qc, 2qc+1
        rope_sincos_fast(__fmul_rn(pf, tail->inv_freq[2 * qc]), v.z, v.x);
        rope_sincos_fast(__fmul_rn(pf, tail->inv_freq[2 * qc + 1]), v.w, v.y);
        *reinterpret_cast<float4*>(cs_buf + p * kCsRow + cs_phys(qc) * 16) = v;
      }
    }
    const int s = it % kStages;
    if (tid == 0 && !mbar_wait_bounded(&tail->full[s], (it / kStages) & 1)) {
      set_status(a.status, kStatusTimeout);
      tail->abort = 1;
    }
    __syncthreads();  // tile t's keys and cos/sin are ready; tile t-1 is retired
    if (tail->abort) return;
    // refill the stage every warp finished with in the previous iteration
    if (tid == 0 && t + kStages - 1 < t_end) issue(t + kStages - 1, (it + kStages - 1) % kStages);

    const uint8_t* st = stages + s * stage_bytes;
#pragma unroll
    for (int i = 0; i < kItemsPerWarp; ++i) {
      if (i >= ipw) break;
      const uint8_t* krow = st + k_off[i];
      const uint4 wl = lds128(krow);
      const uint4 wh = lds128(krow + 128);
      float2 lo[4], hi[4];
      unpack4<T>(wl, lo);
      unpack4<T>(wh, hi);
      float2 kr_lo[4], kr_hi[4];
      if (kRope) {
        const uint8_t* csl = cs_buf + cs_off[i];
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const float4 c = *reinterpret_cast<const float4*>(csl + 16 * m);
          const float2 cc = make_float2(c.x, c.y), ss = make_float2(c.z, c.w);
          const float2 ns = make_float2(-c.z, -c.w);
          kr_lo[m] = __ffma2_rn(hi[m], ss, __fmul2_rn(lo[m], cc));
          kr_hi[m] = __ffma2_rn(lo[m], ns, __fmul2_rn(hi[m], cc));
        }
      } else {
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          kr_lo[m] = lo[m];
          kr_hi[m] = hi[m];
        }
      }
      float v[kMaxR];
#pragma unroll
      for (int r = 0; r < kMaxR; ++r) {
        float2 acc = __fmul2_rn(q_lo[r][0], kr_lo[0]);
#pragma unroll
        for (int m = 1; m < 4; ++m) acc = __ffma2_rn(q_lo[r][m], kr_lo[m], acc);
#pragma unroll
        for (int m = 0; m < 4; ++m) acc = __ffma2_rn(q_hi[r][m], kr_hi[m], acc);
        v[r] = acc.x + acc.y;
      }
      // transposed reduction over the 8 lanes of a key: lanes 2r, 2r+1 end with row r
      const bool b2 = (j & 4) != 0, b1 = (j & 2) != 0;
      const float u0 = (b2 ? v[2] : v[0]) + __shfl_xor_sync(0xffffffffu, b2 ? v[0] : v[2], 4);
      const float u1 = (b2 ? v[3] : v[1]) + __shfl_xor_sync(0xffffffffu, b2 ? v[1] : v[3], 4);
      float w = (b1 ? u1 : u0) + __shfl_xor_sync(0xffffffffu, b1 ? u0 : u1, 2);
      w += __shfl_xor_sync(0xffffffffu, w, 1);
      const int pos = p0 + p_of[i];
      if (writer && pos < a.Sk) out[pos] = int64_t(pos) > vis_limit ? -INFINITY : w;
    }
  }
}

int positions_per_stage(int Hkv) { return min(64, 128 / Hkv); }

size_t g4_smem_bytes(int Hkv, int Tp) {
  return size_t(kStages) * Hkv * Tp * kRowBytes + size_t(2) * Tp * kCsRow + sizeof(G4Tail);
}

template <typename T, bool kRope>
cudaError_t launch_g4(const DecodeArgs& a, int num_sms, cudaStream_t stream) {
  const int Tp = positions_per_stage(a.Hkv);
  const size_t smem = g4_smem_bytes(a.Hkv, Tp);
  auto kern = decode_g4_kernel<T, kRope>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  CUtensorMap kmap;
  e = make_key_tensor_map(&kmap, a.k, std::is_same<T, __nv_bfloat16>::value ? kBF16 : kFP16, a.B,
                          a.Hkv, a.Sk, a.k_sb, a.k_sh, Tp);
  if (e != cudaSuccess) return e;
  DecodeArgs b = a;
  b.ntiles = (a.Sk + Tp - 1) / Tp;
  int ctas = num_sms;
  if (a.B > 1) ctas = (num_sms + a.B - 1) / a.B;
  ctas = max(1, min(ctas, b.ntiles));
  kern<<<dim3(ctas, a.B), kThreads, smem, stream>>>(kmap, b, Tp);
  return cudaGetLastError();
}

}  // namespace

bool decode_g4_supported(const DecodeArgs& a) {
  const int R = a.G * a.sq_n;
  const int H = a.Hkv;
  const bool pow2 = H == 1 || H == 2 || H == 4 || H == 8 || H == 16;
  // 16-byte aligned query rows for the direct vector loads of q
  const bool q_aligned = (reinterpret_cast<uintptr_t>(a.q) & 15u) == 0 && a.q_sb % 8 == 0 &&
                         a.q_sh % 8 == 0 && a.q_ss % 8 == 0;
  return R <= kMaxR && pow2 && q_aligned && g4_smem_bytes(H, positions_per_stage(H)) <= 227 * 1024;
}

cudaError_t launch_decode_scores_g4(const DecodeArgs& a, int dtype, int num_sms,
                                    cudaStream_t stream) {
  const bool rope = a.inv_freq != nullptr;
  if (dtype == kBF16)
    return rope ? launch_g4<__nv_bfloat16, true>(a, num_sms, stream)
                : launch_g4<__nv_bfloat16, false>(a, num_sms, stream);
  return rope ? launch_g4<__half, true>(a, num_sms, stream)
              : launch_g4<__half, false>(a, num_sms, stream);
}

}  // namespace prism
