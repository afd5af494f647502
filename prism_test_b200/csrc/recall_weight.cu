// Value-norm recall weighting (recall_type "qkv" / "qkv2"): every key's score is
// multiplied by the L1 or L2 norm of its value row. ReAttentionMethod.
// _apply_recall_weight (eval_harness/attention_methods/reattention.py:822-842)
// scales the raw key by values.norm(p, dim=-1) before the q·K^T einsum
// (reattention.py:358, reattention_exact.py:547), which is the same product.
// values.norm returns the values' dtype, so the weight is rounded to bf16/fp16
// before it multiplies, as there.
//
// Two passes, both memory-bound:
//   value_norms_kernel streams V once (the only HBM-sized input) and computes
//     the norms on the tensor cores with mma.sync m16n8k16 (bf16 / fp16 in,
//     fp32 accumulate), so the per-element work is one 16-byte load share and
//     no shuffles. A warp takes a task of 32 consecutive keys of one (batch, KV
//     head) as two 16-row tiles; lane (g, t) = (lane / 4, lane % 4) loads the
//     16-byte chunks 4m + t of rows g and g + 8 of each tile, which is an
//     m16n8k16 A fragment up to a permutation of the columns inside each row
//     (harmless: every row is only summed). L1 (qkv): A = |V| (sign bits
//     cleared on the packed words), B = all ones, so every column of D is the
//     row sum. L2 (qkv2): B is the lane's own A registers of rows 0-7 (resp.
//     8-15), so D = V V^T restricted to those columns and its diagonal holds
//     the sums of squares. The products are exact in fp32; the accumulation
//     order differs from a sequential fp32 sum by rounding only.
//     w[(b * Hkv + h) * ld + j] receives the norm rounded to the value dtype.
//   scale_scores_kernel multiplies the fp32 score matrix (still resident in L2
//     after the scorer) by w with float4 accesses, one row per grid row.
//     Masked (-inf) scores stay -inf; a -0 product is written as +0 so that
//     keys of weight 0 tie at +0.
#include "common.cuh"
#include "kernels.h"

namespace prism {
namespace {

constexpr int kNormWarps = 4;

template <typename T>
__device__ __forceinline__ float round_to(float x);
template <>
__device__ __forceinline__ float round_to<__nv_bfloat16>(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}
template <>
__device__ __forceinline__ float round_to<__half>(float x) {
  return __half2float(__float2half_rn(x));
}

// d += A * B for one m16n8k16 tile, 16-bit inputs of type T, fp32 accumulators
template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], uint32_t a0, uint32_t a1,
                                                        uint32_t a2, uint32_t a3, uint32_t b0,
                                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], uint32_t a0, uint32_t a1,
                                                 uint32_t a2, uint32_t a3, uint32_t b0,
                                                 uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <typename T>
constexpr uint32_t kOnes2 = 0;
template <>
constexpr uint32_t kOnes2<__nv_bfloat16> = 0x3f803f80u;  // (1.0, 1.0) in bf16
template <>
constexpr uint32_t kOnes2<__half> = 0x3c003c00u;         // (1.0, 1.0) in fp16

// Two k-steps of one tile from the lane's chunk x of row g and y of row g + 8.
template <typename T, int kP>
__device__ __forceinline__ void tile_steps(float (&d0)[4], float (&d1)[4], uint4 x, uint4 y) {
  if (kP == 1) {
    constexpr uint32_t m = 0x7fff7fffu;
    const uint32_t o = kOnes2<T>;
    mma16816<T>(d0, x.x & m, y.x & m, x.y & m, y.y & m, o, o);
    mma16816<T>(d0, x.z & m, y.z & m, x.w & m, y.w & m, o, o);
  } else {
    mma16816<T>(d0, x.x, y.x, x.y, y.y, x.x, x.y);  // columns = rows 0-7
    mma16816<T>(d1, x.x, y.x, x.y, y.y, y.x, y.y);  // columns = rows 8-15
    mma16816<T>(d0, x.z, y.z, x.w, y.w, x.z, x.w);
    mma16816<T>(d1, x.z, y.z, x.w, y.w, y.z, y.w);
  }
}

// Contiguous 128-wide value rows (v_ss == 128): a persistent kernel, one CTA
// per SM, 12 warps each with its own ring of kRingStages (2) 8 KB stages. Lane 0 of
// a warp refills a stage with one 1-D bulk copy of the task's 32 rows (TMA,
// evict-first), so up to kRingStages tasks per warp are in flight while the
// warp reads the current stage with conflict-free 16-byte shared loads (chunk
// 4m + t + 4 (g & 1) of each row) and runs the same MMAs as value_norms_kernel.
// Each warp walks a contiguous range of tasks, keeping (bh, tile) by increment.
// The norms are gathered so that lane L holds key j0 + L and written coalesced.
// (Weighing the scores in this kernel as well was measured slower than the
// separate scale pass: the read-modify-write of the score rows stalls the
// warp that should be refilling its ring.)
constexpr int kRingWarps = 12;
constexpr int kRingStages = 2;
constexpr int kStageBytes = 32 * 128 * 2;
constexpr int kRingSmem = kRingWarps * kRingStages * kStageBytes + kRingWarps * kRingStages * 8;

template <typename T, int kP>
__global__ void __launch_bounds__(kRingWarps * 32, 1)
    value_norms_ring_kernel(const T* __restrict__ v, int Hkv, int64_t Sk, int64_t v_sb,
                            int64_t v_sh, int64_t ntasks, float* __restrict__ w, int64_t ld,
                            int* status) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  uint8_t* ring = smem + warp * kRingStages * kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kRingWarps * kRingStages * kStageBytes) +
                   warp * kRingStages;
  const int64_t ktiles = (Sk + 31) / 32;
  const int64_t nwarps = int64_t(gridDim.x) * kRingWarps;
  const int64_t gw = int64_t(blockIdx.x) * kRingWarps + warp;
  const int64_t per = ntasks / nwarps, extra = ntasks - per * nwarps;
  const int64_t t_begin = gw * per + (gw < extra ? gw : extra);
  const int64_t count = per + (gw < extra ? 1 : 0);
  if (lane == 0) {
    for (int st = 0; st < kRingStages; ++st) mbar_init(&full[st], 1);
    fence_mbar_init();
  }
  __syncwarp();
  if (count == 0) return;
  const uint64_t pol = l2_policy_evict_first();
  int64_t bh_i = t_begin / ktiles, jt_i = t_begin - (t_begin / ktiles) * ktiles;  // next to issue
  int64_t bh_c = bh_i, jt_c = jt_i;                                            // next to consume
  auto issue = [&](int st) {
    if (lane == 0) {
      const int64_t rows = Sk - jt_i * 32 < 32 ? Sk - jt_i * 32 : 32;
      const int b = int(bh_i / Hkv), h = int(bh_i - int64_t(b) * Hkv);
      const T* src = v + b * v_sb + h * v_sh + jt_i * 32 * 128;
      mbar_arrive_expect_tx(&full[st], uint32_t(rows * 256));
      bulk_g2s(ring + st * kStageBytes, src, uint32_t(rows * 256), &full[st], pol);
    }
    if (++jt_i == ktiles) {
      jt_i = 0;
      ++bh_i;
    }
  };
  const int64_t npro = count < kRingStages ? count : kRingStages;
  for (int st = 0; st < npro; ++st) issue(st);
  const uint32_t ring_u32 = smem_u32(ring);
  const int sw = 4 * (g & 1);
  for (int64_t i = 0; i < count; ++i) {
    const int st = int(i % kRingStages);
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full[st], uint32_t((i / kRingStages) & 1)))) {
      set_status(status, kStatusTimeout);
      return;
    }
    const int64_t rows = Sk - jt_c * 32 < 32 ? Sk - jt_c * 32 : 32;
    const uint32_t base = ring_u32 + st * kStageBytes;
    float d[2][2][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int e = 0; e < 4; ++e) d[a][u][e] = 0.f;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const uint32_t off = uint32_t(((4 * m + t + sw) & 15) * 16);
      uint4 c[4];
#pragma unroll
      for (int r = 0; r < 4; ++r)  // rows g + 8r; rows past the tail read stale bytes
        c[r] = lds128_u32(base + (g + 8 * r) * 256 + off);
      tile_steps<T, kP>(d[0][0], d[0][1], c[0], c[1]);
      tile_steps<T, kP>(d[1][0], d[1][1], c[2], c[3]);
    }
    __syncwarp();  // every lane is done with the stage before it is refilled
    if (i + kRingStages < count) issue(st);
    // norms of rows 16a + g (lo) and 16a + g + 8 (hi), valid in the owner lane
    // of g: t == 0 (L1) or t == g / 2 (L2)
    float nv[2][2];
#pragma unroll
    for (int a = 0; a < 2; ++a) {
      if (kP == 1) {
        nv[a][0] = d[a][0][0];
        nv[a][1] = d[a][0][2];
      } else {
        nv[a][0] = sqrtf((g & 1) ? d[a][0][1] : d[a][0][0]);
        nv[a][1] = sqrtf((g & 1) ? d[a][1][3] : d[a][1][2]);
      }
    }
    // lane L takes row L = 16 a' + 8 hi' + g' from the owner lane of g'
    const int gl = lane & 7, src = gl * 4 + (kP == 1 ? 0 : gl >> 1);
    const float n00 = __shfl_sync(0xffffffffu, nv[0][0], src);
    const float n01 = __shfl_sync(0xffffffffu, nv[0][1], src);
    const float n10 = __shfl_sync(0xffffffffu, nv[1][0], src);
    const float n11 = __shfl_sync(0xffffffffu, nv[1][1], src);
    const float wl = round_to<T>(lane < 16 ? (lane < 8 ? n00 : n01) : (lane < 24 ? n10 : n11));
    if (lane < rows) w[bh_c * ld + jt_c * 32 + lane] = wl;
    if (++jt_c == ktiles) {
      jt_c = 0;
      ++bh_c;
    }
  }
}

template <typename T, int kP>
__global__ void __launch_bounds__(kNormWarps * 32)
    value_norms_kernel(const T* __restrict__ v, int B, int Hkv, int64_t Sk, int64_t v_sb,
                       int64_t v_sh, int64_t v_ss, int Dv, float* __restrict__ w, int64_t ld) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int nchunks = Dv / 8;  // 16-byte chunks per row
  const int64_t ktiles = (Sk + 31) / 32;
  const int64_t ntasks = int64_t(B) * Hkv * ktiles;
  for (int64_t task = int64_t(blockIdx.x) * kNormWarps + warp; task < ntasks;
       task += int64_t(gridDim.x) * kNormWarps) {
    const int64_t bh = task / ktiles, j0 = (task - bh * ktiles) * 32;
    const int b = int(bh / Hkv), h = int(bh - int64_t(b) * Hkv);
    const T* vb = v + b * v_sb + h * v_sh;
    // rows of this lane: tile 0 -> j0 + g, j0 + g + 8; tile 1 -> + 16
    const T* rp[4];
    bool ok[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int64_t j = j0 + g + 8 * r;
      ok[r] = j < Sk;
      rp[r] = vb + (ok[r] ? j : 0) * v_ss;
    }
    float d[2][2][4];  // [tile][diag block][fragment]
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int e = 0; e < 4; ++e) d[i][u][e] = 0.f;
    for (int cb = 0; cb < nchunks; cb += 16) {
      uint4 c[4][4];  // [row][m]
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const int ch = cb + 4 * m + t;
          c[r][m] = ok[r] && ch < nchunks ? __ldcs(reinterpret_cast<const uint4*>(rp[r] + ch * 8))
                                          : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        tile_steps<T, kP>(d[0][0], d[0][1], c[0][m], c[1][m]);
        tile_steps<T, kP>(d[1][0], d[1][1], c[2][m], c[3][m]);
      }
    }
    // row g of tile i: L1 -> d[i][0][0] in every lane of the quad; L2 -> the
    // diagonal element D[g][g], held by lane t == g / 2 in d[i][0][g & 1];
    // row g + 8: L1 -> d[i][0][2]; L2 -> D[g+8][g] of the second block, in
    // d[i][1][2 + (g & 1)] of lane t == g / 2
    if (kP == 1 ? t == 0 : t == (g >> 1)) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        float lo, hi;
        if (kP == 1) {
          lo = d[i][0][0];
          hi = d[i][0][2];
        } else {
          lo = sqrtf((g & 1) ? d[i][0][1] : d[i][0][0]);
          hi = sqrtf((g & 1) ? d[i][1][3] : d[i][1][2]);
        }
        const int64_t j = j0 + 16 * i + g;
        if (j < Sk) w[bh * ld + j] = round_to<T>(lo);
        if (j + 8 < Sk) w[bh * ld + j + 8] = round_to<T>(hi);
      }
    }
  }
}

__device__ __forceinline__ float weigh(float x, float w) {
  return x != -INFINITY ? x * w + 0.0f : x;
}

// scores [rows, ld] with rows ordered (b, hq, s); w [B * Hkv, ld]; ld % 4 == 0.
// blockIdx.x: a span of kScaleVec * 4 * blockDim.x columns (each thread takes
// kScaleVec float4 at a stride of blockDim.x, all loads issued before the
// stores); blockIdx.y (+ multiples of gridDim.y): the row, so the row's weight
// row is found once per block.
constexpr int kScaleVec = 4;
__global__ void __launch_bounds__(256) scale_scores_kernel(float* __restrict__ scores, int rows,
                                                           int64_t Sk, int64_t ld, int Hq, int G,
                                                           int Sq, int Hkv,
                                                           const float* __restrict__ w) {
  const int64_t q4 = ld / 4;
  const int64_t c0 = int64_t(blockIdx.x) * blockDim.x * kScaleVec + threadIdx.x;
  for (int row = blockIdx.y; row < rows; row += gridDim.y) {
    const int bhq = row / Sq;
    const int b = bhq / Hq, hq = bhq - b * Hq;
    float4* sp = reinterpret_cast<float4*>(scores + int64_t(row) * ld);
    const float4* wp = reinterpret_cast<const float4*>(w + (int64_t(b) * Hkv + hq / G) * ld);
    float4 x[kScaleVec], wv[kScaleVec];
#pragma unroll
    for (int u = 0; u < kScaleVec; ++u) {
      const int64_t c = c0 + int64_t(u) * blockDim.x;
      if (c < q4) {
        x[u] = sp[c];
        wv[u] = wp[c];
      }
    }
#pragma unroll
    for (int u = 0; u < kScaleVec; ++u) {
      const int64_t c = c0 + int64_t(u) * blockDim.x;
      if (c < q4) {
        const int64_t j = 4 * c;
        float4 y = x[u];
        y.x = weigh(y.x, wv[u].x);
        if (j + 1 < Sk) y.y = weigh(y.y, wv[u].y);
        if (j + 2 < Sk) y.z = weigh(y.z, wv[u].z);
        if (j + 3 < Sk) y.w = weigh(y.w, wv[u].w);
        sp[c] = y;
      }
    }
  }
}

}  // namespace

size_t weight_workspace_bytes(int64_t B, int64_t Hkv, int64_t Sk) {
  const int64_t ld = (Sk + 3) / 4 * 4;
  return (size_t(B) * size_t(Hkv) * size_t(ld) * sizeof(float) + 255) / 256 * 256;
}

template <typename T, int kP>
cudaError_t launch_ring(const WeightArgs& a, int64_t ntasks, int num_sms, cudaStream_t stream) {
  cudaError_t e = cudaFuncSetAttribute(value_norms_ring_kernel<T, kP>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, kRingSmem);
  if (e != cudaSuccess) return e;
  const int64_t want = (ntasks + kRingWarps - 1) / kRingWarps;
  const int grid = int(want < num_sms ? want : num_sms);
  value_norms_ring_kernel<T, kP><<<grid, kRingWarps * 32, kRingSmem, stream>>>(
      static_cast<const T*>(a.v), a.Hkv, a.Sk, a.v_sb, a.v_sh, ntasks, a.w, a.ld, a.status);
  return cudaGetLastError();
}

cudaError_t launch_value_norms(const WeightArgs& a, int dtype, int num_sms, cudaStream_t stream) {
  const int64_t ntasks = int64_t(a.B) * a.Hkv * ((a.Sk + 31) / 32);
  if (a.Dv == 128 && a.v_ss == 128) {
    if (dtype == kBF16)
      return a.p == 1 ? launch_ring<__nv_bfloat16, 1>(a, ntasks, num_sms, stream)
                      : launch_ring<__nv_bfloat16, 2>(a, ntasks, num_sms, stream);
    return a.p == 1 ? launch_ring<__half, 1>(a, ntasks, num_sms, stream)
                    : launch_ring<__half, 2>(a, ntasks, num_sms, stream);
  }
  const int64_t want = (ntasks + kNormWarps - 1) / kNormWarps;
  const int grid = int(want < int64_t(num_sms) * 5 ? want : int64_t(num_sms) * 5);
  const dim3 block(kNormWarps * 32);
  if (dtype == kBF16) {
    auto* v = static_cast<const __nv_bfloat16*>(a.v);
    if (a.p == 1)
      value_norms_kernel<__nv_bfloat16, 1><<<grid, block, 0, stream>>>(v, a.B, a.Hkv, a.Sk, a.v_sb, a.v_sh, a.v_ss, a.Dv, a.w, a.ld);
    else
      value_norms_kernel<__nv_bfloat16, 2><<<grid, block, 0, stream>>>(v, a.B, a.Hkv, a.Sk, a.v_sb, a.v_sh, a.v_ss, a.Dv, a.w, a.ld);
  } else {
    auto* v = static_cast<const __half*>(a.v);
    if (a.p == 1)
      value_norms_kernel<__half, 1><<<grid, block, 0, stream>>>(v, a.B, a.Hkv, a.Sk, a.v_sb, a.v_sh, a.v_ss, a.Dv, a.w, a.ld);
    else
      value_norms_kernel<__half, 2><<<grid, block, 0, stream>>>(v, a.B, a.Hkv, a.Sk, a.v_sb, a.v_sh, a.v_ss, a.Dv, a.w, a.ld);
  }
  return cudaGetLastError();
}

cudaError_t launch_scale_scores(const WeightArgs& a, int num_sms, cudaStream_t stream) {
  (void)num_sms;
  const int rows = a.B * a.Hq * a.Sq;
  const int64_t cblocks = (a.ld / 4 + 256 * kScaleVec - 1) / (256 * kScaleVec);
  const dim3 grid(unsigned(cblocks), unsigned(rows < 65535 ? rows : 65535));
  scale_scores_kernel<<<grid, 256, 0, stream>>>(a.scores, rows, a.Sk, a.ld, a.Hq, a.G, a.Sq, a.Hkv, a.w);
  return cudaGetLastError();
}

}  // namespace prism
