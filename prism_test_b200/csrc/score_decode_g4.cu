// Decode scorer, fast path for at most 4 query rows per KV head (GQA decode:
// Hq/Hkv <= 4 query heads per KV head, one query position) — the common decode
// shape of the reference's recall (reattention.py:486-498 with q_len = 1).
//
// Same math as score_decode.cu (inverse RoPE fused into the key load, fp32
// dot products), laid out so that shared memory is not the bottleneck:
//
//  * a stage holds Tp key positions of EVERY KV head of one batch row (one
//    bulk copy per head, one mbarrier, <= 32 KB), four stages: three tiles are
//    in flight while one is consumed. There is no separate producer warp (it
//    would cap the CTA at 168 registers): thread 0 issues the copies of tile
//    t+3 right after the per-tile barrier, which proves that every warp has
//    finished tile t-1 and its stage is free;
//  * each consumer warp owns work items (kv head, 8 positions); items are dealt
//    head-major in contiguous ranges so a warp keeps its head's query rows in
//    registers (4 rows x 32 dims per lane) instead of re-reading them per key;
//  * the RoPE cos/sin of a tile (Tp positions x 64 frequencies) is computed
//    once by all consumer threads into a double-buffered shared table and read
//    by every head's warp;
//  * 4 lanes share a key (32 dims each). Lanes of odd positions load their key
//    and table chunks in a rotated order, so every 8-lane phase of a 128-bit
//    shared load touches 8 distinct bank groups (no conflicts), and the
//    table is stored with a matching XOR/rotate swizzle;
//  * rotation and dot products use packed fp32x2 FMA (__ffma2_rn / __fmul2_rn).
#include "common.cuh"
#include "kernels.h"
#include "rope_sincos.cuh"

namespace prism {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers;
constexpr int kStages = 4;
constexpr int kMaxR = 4;
constexpr int kMaxStageBytes = 32 * 1024;

struct __align__(16) G4Tail {
  uint64_t full[kStages];
  float inv_freq[64];
};

// physical 16-byte chunk of logical chunk q (0..31) of the cos/sin row of
// position p: rotates each group of 8 chunks by 2*(q/8) + (p&1)
__device__ __forceinline__ int cs_phys(int p, int q) {
  return (q & ~7) | (((q & 7) + 2 * (q >> 3) + (p & 1)) & 7);
}

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
  uint8_t* cs_tab = smem + kStages * stage_bytes;            // [2][Tp][512 B]
  float* q_s = reinterpret_cast<float*>(cs_tab + 2 * Tp * 512);  // [Hkv][R][128]
  G4Tail* tail = reinterpret_cast<G4Tail*>(q_s + size_t(rows) * kHeadDim);

  const int tid = threadIdx.x;
  const int b = blockIdx.y;
  const int t_begin = static_cast<int>(int64_t(blockIdx.x) * a.ntiles / gridDim.x);
  const int t_end = static_cast<int>(int64_t(blockIdx.x + 1) * a.ntiles / gridDim.x);

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

  const int warp = tid >> 5, lane = tid & 31;
  const uint8_t* kb = static_cast<const uint8_t*>(a.k) + int64_t(b) * a.k_sb * int64_t(sizeof(T));
  const uint64_t pol = l2_policy_evict_first();
  // issue the bulk copies of tile t into stage s (thread 0 only)
  auto issue = [&](int t, int s) {
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

  // ---------------- consumers ----------------------------------------------------
  const int j = lane & 3;          // dim slice: [16j, 16j+16) and [64+16j, 64+16j+16)
  const int pl = lane >> 2;        // position within an item (0..7)
  const int par = pl & 1;          // rotated chunk order for odd positions
  const int npass = Tp / 8;
  const int nitems = Hkv * npass;  // head-major: item i -> head i / npass, pass i % npass
  const int i_begin = warp * nitems / kConsumerWarps;
  const int i_end = (warp + 1) * nitems / kConsumerWarps;

  // this lane's slot u (0..15) holds dim 16j + ((u + 8*par) & 15) of each half
  float2 qreg[kMaxR][16];  // [row][slot pair]: pairs 0..3 lo slots 0..7, 4..7 lo 8..15, 8..15 hi
  int q_head = -1;

  int it = 0;
  for (int t = t_begin; t < t_end; ++t, ++it) {
    const int p0 = t * Tp;
    uint8_t* cs_buf = cs_tab + (it & 1) * Tp * 512;
    if (kRope) {
      for (int idx = tid; idx < Tp * 32; idx += kConsumers) {
        const int p = idx >> 5, qc = idx & 31;
        const float pf = static_cast<float>(a.pos_offset + p0 + p);
        float4 v;
        rope_sincos(__fmul_rn(pf, tail->inv_freq[2 * qc]), v.z, v.x);
        rope_sincos(__fmul_rn(pf, tail->inv_freq[2 * qc + 1]), v.w, v.y);
        // chunk = (cos f0, cos f1, sin f0, sin f1)
        *reinterpret_cast<float4*>(cs_buf + p * 512 + cs_phys(p, qc) * 16) = v;
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
    for (int item = i_begin; item < i_end; ++item) {
      const int h = item / npass;
      const int pass = item % npass;
      if (h != q_head) {
        q_head = h;
        const float* qh = q_s + size_t(h) * R * kHeadDim;
#pragma unroll
        for (int r = 0; r < kMaxR; ++r) {
          const float* qr = qh + min(r, R - 1) * kHeadDim;
#pragma unroll
          for (int u2 = 0; u2 < 8; ++u2) {
            const int d = 16 * j + ((2 * u2 + 8 * par) & 15);
            qreg[r][u2] = *reinterpret_cast<const float2*>(qr + d);
            qreg[r][8 + u2] = *reinterpret_cast<const float2*>(qr + 64 + d);
          }
        }
      }
      const int p = pass * 8 + pl;  // position within the tile
      const uint8_t* krow = st + (size_t(h) * Tp + p) * kRowBytes;
      const uint8_t* csrow = cs_buf + p * 512;
      float2 acc[kMaxR];
#pragma unroll
      for (int r = 0; r < kMaxR; ++r) acc[r] = make_float2(0.f, 0.f);
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        // slots 8hf .. 8hf+7: byte offset of this half-slice inside the 32-byte slice
        const int off = 16 * ((hf + par) & 1);
        const uint4 wl = lds128(krow + 32 * j + off);
        const uint4 wh = lds128(krow + 128 + 32 * j + off);
        float2 lo[4], hi[4];
        unpack4<T>(wl, lo);
        unpack4<T>(wh, hi);
        float2 kr_lo[4], kr_hi[4];
        if (kRope) {
#pragma unroll
          for (int m = 0; m < 2; ++m) {
            // table chunk for slot pairs (4hf + 2m, 4hf + 2m + 1): logical chunk
            // 8j + ((4hf + 2m + 4par) & 7) and the next one
            const int lc0 = 8 * j + ((4 * hf + 2 * m + 4 * par) & 7);
            const int lc1 = 8 * j + ((4 * hf + 2 * m + 1 + 4 * par) & 7);
            const float4 c0 = *reinterpret_cast<const float4*>(csrow + cs_phys(p, lc0) * 16);
            const float4 c1 = *reinterpret_cast<const float4*>(csrow + cs_phys(p, lc1) * 16);
            const float2 cc0 = make_float2(c0.x, c0.y), ss0 = make_float2(c0.z, c0.w);
            const float2 cc1 = make_float2(c1.x, c1.y), ss1 = make_float2(c1.z, c1.w);
            const float2 ns0 = make_float2(-c0.z, -c0.w), ns1 = make_float2(-c1.z, -c1.w);
            kr_lo[2 * m] = __ffma2_rn(hi[2 * m], ss0, __fmul2_rn(lo[2 * m], cc0));
            kr_hi[2 * m] = __ffma2_rn(lo[2 * m], ns0, __fmul2_rn(hi[2 * m], cc0));
            kr_lo[2 * m + 1] = __ffma2_rn(hi[2 * m + 1], ss1, __fmul2_rn(lo[2 * m + 1], cc1));
            kr_hi[2 * m + 1] = __ffma2_rn(lo[2 * m + 1], ns1, __fmul2_rn(hi[2 * m + 1], cc1));
          }
        } else {
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            kr_lo[m] = lo[m];
            kr_hi[m] = hi[m];
          }
        }
#pragma unroll
        for (int r = 0; r < kMaxR; ++r) {
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            acc[r] = __ffma2_rn(qreg[r][4 * hf + m], kr_lo[m], acc[r]);
            acc[r] = __ffma2_rn(qreg[r][8 + 4 * hf + m], kr_hi[m], acc[r]);
          }
        }
      }
      // lane j ends with the full sum of row j (transposed quad reduction)
      float v[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) v[r] = acc[r].x + acc[r].y;
      const bool b1 = (j & 2) != 0, b0 = (j & 1) != 0;
      float u2v[2];
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        const float send = b1 ? v[m] : v[m + 2];
        const float keep = b1 ? v[m + 2] : v[m];
        u2v[m] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
      }
      const float send = b0 ? u2v[0] : u2v[1];
      const float keep = b0 ? u2v[1] : u2v[0];
      const float sum = keep + __shfl_xor_sync(0xffffffffu, send, 1);
      const int pos = p0 + p;
      if (j < R && pos < a.Sk) {
        const int gi = j / a.sq_n, sl = j % a.sq_n;
        const int s_abs = a.s0 + sl;
        const int64_t row = (int64_t(b) * a.Hq + h * a.G + gi) * a.Sq + s_abs;
        float val = sum;
        if (a.causal && int64_t(pos) > a.causal_offset + s_abs) val = -INFINITY;
        a.scores[row * a.ld + pos] = val;
      }
    }
  }
}

int positions_per_stage(int Hkv) {
  // stage = Hkv * Tp * 256 B <= 32 KB, Tp a multiple of 8 (one item), at most 64
  int tp = kMaxStageBytes / (Hkv * kRowBytes);
  tp = tp > 64 ? 64 : tp;
  return tp & ~7;
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
  if (R > kMaxR || a.Hkv > 16) return false;
  const int Tp = positions_per_stage(a.Hkv);
  return g4_smem_bytes(a.Hkv, a.Hkv * R, Tp) <= 227 * 1024;
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
