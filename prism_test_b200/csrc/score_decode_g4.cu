// Decode scorer, fast path for at most 4 query rows per KV head (GQA decode:
// Hq/Hkv <= 4 query heads per KV head at one query position) — the decode
// shape of the reference's recall (reattention.py:486-498 with q_len = 1).
//
// Same math as score_decode.cu (inverse RoPE fused into the key load, fp32
// dot products), organised for issue rate and shared-memory bandwidth:
//
//  * a stage holds Tp key positions of EVERY KV head of one batch row (one TMA
//    bulk copy per head, one mbarrier, <= 32 KB); four stages, three tiles in
//    flight while one is consumed. Thread 0 issues the copies of tile t+3 right
//    after the per-tile barrier, which proves every warp is done with tile t-1;
//  * 16 warps; a work item is (kv head, 4 positions), 8 lanes per key, each
//    lane 8 rotation pairs (dims [8j, 8j+8) and [64+8j, 64+8j+8)). Items are
//    dealt head-major in contiguous ranges so a warp keeps its head's query
//    rows in registers (4 rows x 16 values per lane);
//  * the RoPE cos/sin of a tile (Tp positions x 64 frequencies) is computed
//    once by all threads into a double-buffered shared table, stored with a
//    rotation swizzle so each 8-lane phase of a 128-bit load hits 8 distinct
//    bank groups (key rows are read conflict-free as laid out);
//  * rotation and dot products in packed fp32x2 FMA (__ffma2_rn / __fmul2_rn),
//    two accumulator chains per row.
#include "common.cuh"
#include "kernels.h"
#include "rope_sincos.cuh"

namespace prism {
namespace {

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kStages = 4;
constexpr int kMaxR = 4;
constexpr int kMaxStageBytes = 32 * 1024;

struct __align__(16) G4Tail {
  uint64_t full[kStages];
  float inv_freq[64];
};

// physical 16-byte chunk of logical chunk q (0..31) in a position's cos/sin row:
// each group of 8 chunks is rotated by q/8
__device__ __forceinline__ int cs_phys(int q) { return (q & ~7) | (((q & 7) + (q >> 3)) & 7); }

template <typename T>
__device__ __forceinline__ void unpack4(const uint4& v, float2 out[4]) {
  Unpack<T>::run(v.x, out[0].x, out[0].y);
  Unpack<T>::run(v.y, out[1].x, out[1].y);
  Unpack<T>::run(v.z, out[2].x, out[2].y);
  Unpack<T>::run(v.w, out[3].x, out[3].y);
}

template <typename T, bool kRope>
__global__ void __launch_bounds__(kThreads, 1) decode_g4_kernel(const DecodeArgs a, int Tp) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int Hkv = a.Hkv;
  const int R = a.G * a.sq_n;  // <= 4
  const int rows = Hkv * R;
  const size_t stage_bytes = size_t(Hkv) * Tp * kRowBytes;
  uint8_t* stages = smem;
  uint8_t* cs_tab = smem + kStages * stage_bytes;                // [2][Tp][512 B]
  float* q_s = reinterpret_cast<float*>(cs_tab + 2 * Tp * 512);  // [Hkv][R][128]
  G4Tail* tail = reinterpret_cast<G4Tail*>(q_s + size_t(rows) * kHeadDim);

  const int tid = threadIdx.x;
  const int b = blockIdx.y;
  const int t_begin = static_cast<int>(int64_t(blockIdx.x) * a.ntiles / gridDim.x);
  const int t_end = static_cast<int>(int64_t(blockIdx.x + 1) * a.ntiles / gridDim.x);

  // let the selection kernel (launched with programmatic stream serialization)
  // be scheduled while this grid drains; it waits for our completion itself
  asm volatile("griddepcontrol.launch_dependents;");
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&tail->full[s], 1);
    fence_mbar_init();
  }
  const T* qg = static_cast<const T*>(a.q);
  for (int e = tid; e < rows * kHeadDim; e += kThreads) {
    const int row = e / kHeadDim, d = e % kHeadDim;
    const int hk = row / R, r = row % R;
    const int gi = r / a.sq_n, sl = r % a.sq_n;
    q_s[e] = to_f32(qg[int64_t(b) * a.q_sb + int64_t(hk * a.G + gi) * a.q_sh +
                       int64_t(a.s0 + sl) * a.q_ss + d]);
  }
  if (kRope) {
    for (int i = tid; i < kHeadDim / 2; i += kThreads) tail->inv_freq[i] = a.inv_freq[i];
  }
  __syncthreads();

  const uint8_t* kb = static_cast<const uint8_t*>(a.k) + int64_t(b) * a.k_sb * int64_t(sizeof(T));
  // bulk copies of tile t into stage s (thread 0 only)
  auto issue = [&](int t, int s) {
    const uint64_t pol = l2_policy_evict_first();
    const int p0 = t * Tp;
    const int nvalid = min(Tp, a.Sk - p0);
    const uint32_t bytes = uint32_t(nvalid) * kRowBytes;
    mbar_arrive_expect_tx(&tail->full[s], bytes * uint32_t(Hkv));
    uint8_t* dst = stages + s * stage_bytes;
    for (int h = 0; h < Hkv; ++h)
      bulk_g2s(dst + size_t(h) * Tp * kRowBytes,
               kb + (int64_t(h) * a.k_sh + int64_t(p0) * kHeadDim) * int64_t(sizeof(T)), bytes,
               &tail->full[s], pol);
  };
  if (tid == 0) {
    for (int k = 0; k < kStages - 1 && t_begin + k < t_end; ++k) issue(t_begin + k, k);
  }

  const int warp = tid >> 5, lane = tid & 31;
  const int j = lane & 7;    // rotation pairs [8j, 8j+8)
  const int pl = lane >> 3;  // position within an item (0..3)
  const int npass = Tp / 4;
  const int nitems = Hkv * npass;  // item i -> head i / npass, positions 4*(i % npass) ..
  const int i_begin = warp * nitems / kWarps;
  const int i_end = (warp + 1) * nitems / kWarps;
  // byte offsets of this lane's 4 cos/sin chunks inside a position row
  int cs_off[4];
#pragma unroll
  for (int m = 0; m < 4; ++m) cs_off[m] = cs_phys(4 * j + m) * 16;

  float2 q_lo[kMaxR][4], q_hi[kMaxR][4];  // dims 8j+2m, 8j+2m+1 (and +64)
  int q_head = -1;
  // first item's (head, pass); later items advance incrementally (no divisions
  // in the loop)
  const int h_begin = i_begin / npass, pass_begin = i_begin % npass;
  // output row of this lane (row r = j/2 of the head's group), minus the head term
  const int r_lane = j >> 1;
  const int gi_lane = r_lane / a.sq_n, s_abs_lane = a.s0 + r_lane % a.sq_n;
  const bool writer = (j & 1) == 0 && r_lane < R;
  const int64_t row_lane = int64_t(b) * a.Hq * a.Sq + int64_t(gi_lane) * a.Sq + s_abs_lane;
  const int64_t vis_limit = a.causal ? a.causal_offset + s_abs_lane : INT64_MAX;
  float* out_row = nullptr;

  int it = 0;
  for (int t = t_begin; t < t_end; ++t, ++it) {
    const int p0 = t * Tp;
    uint8_t* cs_buf = cs_tab + (it & 1) * Tp * 512;
    if (kRope) {
      for (int idx = tid; idx < Tp * 32; idx += kThreads) {
        const int p = idx >> 5, qc = idx & 31;
        const float pf = static_cast<float>(a.pos_offset + p0 + p);
        float4 v;  // (cos f0, cos f1, sin f0, sin f1) of freqs 2qc, 2qc+1
        rope_sincos_fast(__fmul_rn(pf, tail->inv_freq[2 * qc]), v.z, v.x);
        rope_sincos_fast(__fmul_rn(pf, tail->inv_freq[2 * qc + 1]), v.w, v.y);
        *reinterpret_cast<float4*>(cs_buf + p * 512 + cs_phys(qc) * 16) = v;
      }
    }
    __syncthreads();  // cos/sin of tile t ready; every warp is done with tile t-1
    if (tid == 0 && t + kStages - 1 < t_end) issue(t + kStages - 1, (it + kStages - 1) % kStages);

    const int s = it % kStages;
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&tail->full[s], (it / kStages) & 1))) {
      set_status(a.status, kStatusTimeout);
      return;
    }
    const uint8_t* st = stages + s * stage_bytes;
    int h = h_begin, pass = pass_begin;
    for (int item = i_begin; item < i_end; ++item) {
      if (h != q_head) {
        q_head = h;
        out_row = a.scores + (row_lane + int64_t(h) * a.G * a.Sq) * a.ld;
        const float* qh = q_s + size_t(h) * R * kHeadDim;
#pragma unroll
        for (int r = 0; r < kMaxR; ++r) {
          const float* qr = qh + min(r, R - 1) * kHeadDim + 8 * j;
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            q_lo[r][m] = *reinterpret_cast<const float2*>(qr + 2 * m);
            q_hi[r][m] = *reinterpret_cast<const float2*>(qr + 64 + 2 * m);
          }
        }
      }
      const int p = 4 * pass + pl;  // position within the tile
      const uint8_t* krow = st + (size_t(h) * Tp + p) * kRowBytes;
      if (++pass == npass) {  // advance to the next item's (head, pass)
        pass = 0;
        ++h;
      }
      const uint4 wl = lds128(krow + 16 * j);
      const uint4 wh = lds128(krow + 128 + 16 * j);
      float2 lo[4], hi[4];
      unpack4<T>(wl, lo);
      unpack4<T>(wh, hi);
      float2 kr_lo[4], kr_hi[4];
      if (kRope) {
        const uint8_t* csrow = cs_buf + p * 512;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const float4 c = *reinterpret_cast<const float4*>(csrow + cs_off[m]);
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
        float2 a0 = __fmul2_rn(q_lo[r][0], kr_lo[0]);
        float2 a1 = __fmul2_rn(q_hi[r][0], kr_hi[0]);
#pragma unroll
        for (int m = 1; m < 4; ++m) {
          a0 = __ffma2_rn(q_lo[r][m], kr_lo[m], a0);
          a1 = __ffma2_rn(q_hi[r][m], kr_hi[m], a1);
        }
        const float2 a2 = __fadd2_rn(a0, a1);
        v[r] = a2.x + a2.y;
      }
      // transposed reduction over the 8 lanes of a key: lanes 2r, 2r+1 end with row r
      const bool b2 = (j & 4) != 0, b1 = (j & 2) != 0;
      const float u0 = (b2 ? v[2] : v[0]) + __shfl_xor_sync(0xffffffffu, b2 ? v[0] : v[2], 4);
      const float u1 = (b2 ? v[3] : v[1]) + __shfl_xor_sync(0xffffffffu, b2 ? v[1] : v[3], 4);
      float w = (b1 ? u1 : u0) + __shfl_xor_sync(0xffffffffu, b1 ? u0 : u1, 2);
      w += __shfl_xor_sync(0xffffffffu, w, 1);
      const int pos = p0 + p;
      if (writer && pos < a.Sk) out_row[pos] = int64_t(pos) > vis_limit ? -INFINITY : w;
    }
  }
}

int positions_per_stage(int Hkv) {
  // stage = Hkv * Tp * 256 B <= 32 KB, Tp a multiple of 4 (one item), at most 64
  int tp = kMaxStageBytes / (Hkv * kRowBytes);
  tp = tp > 64 ? 64 : tp;
  return tp & ~3;
}

size_t g4_smem_bytes(int Hkv, int rows, int Tp) {
  return size_t(kStages) * Hkv * Tp * kRowBytes + size_t(2) * Tp * 512 +
         size_t(rows) * kHeadDim * sizeof(float) + sizeof(G4Tail);
}

template <typename T, bool kRope>
cudaError_t launch_g4(const DecodeArgs& a, int num_sms, cudaStream_t stream) {
  const int Tp = positions_per_stage(a.Hkv);
  const int rows = a.Hkv * a.G * a.sq_n;
  const size_t smem = g4_smem_bytes(a.Hkv, rows, Tp);
  auto kern = decode_g4_kernel<T, kRope>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  DecodeArgs b = a;
  b.ntiles = (a.Sk + Tp - 1) / Tp;
  int ctas = num_sms;
  if (a.B > 1) ctas = (num_sms + a.B - 1) / a.B;
  ctas = max(1, min(ctas, b.ntiles));
  kern<<<dim3(ctas, a.B), kThreads, smem, stream>>>(b, Tp);
  return cudaGetLastError();
}

}  // namespace

bool decode_g4_supported(const DecodeArgs& a) {
  const int R = a.G * a.sq_n;
  if (R > kMaxR || a.Hkv > 32) return false;
  const int Tp = positions_per_stage(a.Hkv);
  return Tp >= 4 && g4_smem_bytes(a.Hkv, a.Hkv * R, Tp) <= 227 * 1024;
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
