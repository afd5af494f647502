// Decode scorer on register tensor-core tiles: the inverse RoPE rotation of the
// keys stays on the fp32 CUDA cores (fused into the key load, as in
// score_decode.cu), and the q·K^T dot products of up to 8 (or 16) query rows
// per KV head are mma.sync m16n8k8 TF32 tiles fed straight from registers:
// A = 16 rotated keys x 8 dims, B = 8 dims x 8 query rows, fp32 accumulate.
// This replaces ~1300 CUDA-core instructions per (key, KV head) — unpack,
// 4-row FMA chains, an 8-lane shuffle reduction — by ~550.
//
// Reference path: ReAttentionMethod._unrotate_keys + _dense_topk's einsum
// (eval_harness/attention_methods/reattention.py:743-793, 486-498).
//
// Precision: the tensor core truncates a TF32 operand to its top 19 bits. The
// cos/sin table is scaled by (1 + 2^-11), so a rotated key k_raw = m * 2^e
// (1 <= m < 2) gains m/2 TF32 ulps before the truncation and enters the MMA
// within a relative 2^-11 of k_raw (the round-to-nearest bound, without a
// per-element rounding instruction). bf16/fp16 queries and un-rotated keys are
// exact in TF32; products and sums are fp32. The score error is at most
// 2^-11 * sum_i |q_i k_i| <= 0.49 of the 1e-3 * ||q|| ||k|| tolerance.
//
// Layout and scheduling:
//  * a stage = Tp key positions of every KV head of a batch row, one tiled TMA
//    copy (4-D tensor map, box {128, Tp, Hkv, 1}), 32 KB; four stages, three
//    tiles in flight; Tp = 128 / Hkv so a tile holds 8 items of 16 keys x 1
//    head, one per warp (8 warps);
//  * per tile all threads compute the cos/sin of Tp positions x 64 frequencies
//    into a double-buffered shared table; thread 0 issues tile t+3 and alone
//    waits for tile t; the block barrier publishes both;
//  * lane (g, c) of a warp owns keys g and g+8 of the item and rotation pairs
//    [16c, 16c+16) of both halves — exactly the A-fragment slots (k-columns c
//    and c+4 of each k-step) once dims are assigned to k-steps as
//    step s < 8: dims 16c+2s, 16c+2s+1; step s >= 8: dims 64+16c+2(s-8), +1;
//    the B fragment (query rows) uses the same assignment;
//  * the cos/sin table places lane c's 128-byte block at 144*c in a 576-byte
//    position row, so the 8 lanes of a 128-bit load phase (2 keys x 4 c) hit 8
//    distinct bank groups.
#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "rope_sincos.cuh"
#include "tensor_map.h"

namespace prism {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kStages = 4;
constexpr int kCsRow = 576;   // bytes per position in the cos/sin table
constexpr int kCsLane = 144;  // bytes between consecutive lanes' 128-byte blocks

struct __align__(16) MmaTail {
  uint64_t full[kStages];
  float inv_freq[64];
  int abort;
};

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& v, float2 out[4]) {
  Unpack<T>::run(v.x, out[0].x, out[0].y);
  Unpack<T>::run(v.y, out[1].x, out[1].y);
  Unpack<T>::run(v.z, out[2].x, out[2].y);
  Unpack<T>::run(v.w, out[3].x, out[3].y);
}

__device__ __forceinline__ void mma_tf32(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// kNT n-tiles of 8 query rows (R <= 8 * kNT)
template <typename T, bool kRope, int kNT>
__global__ void __launch_bounds__(kThreads, 1)
    decode_mma_kernel(const __grid_constant__ CUtensorMap kmap, const DecodeArgs a, int Tp) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int Hkv = a.Hkv;
  const int R = a.G * a.sq_n;
  const uint32_t stage_bytes = uint32_t(Hkv) * Tp * kRowBytes;
  uint8_t* stages = smem;
  uint8_t* cs_tab = smem + kStages * stage_bytes;  // [2][Tp][kCsRow]
  MmaTail* tail = reinterpret_cast<MmaTail*>(cs_tab + 2 * Tp * kCsRow);

  const int tid = threadIdx.x;
  const int b = blockIdx.y;
  const int t_begin = static_cast<int>(int64_t(blockIdx.x) * a.ntiles / gridDim.x);
  const int t_end = static_cast<int>(int64_t(blockIdx.x + 1) * a.ntiles / gridDim.x);

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

  // ---- per-lane constants ----------------------------------------------------------
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2;  // keys g and g+8 of the item; query row g of each n-tile
  const int c = lane & 3;   // rotation pairs [16c, 16c+16)
  const int nks = Tp / 16;  // 16-key slices per head in a tile
  const int h = warp / nks;
  const int key0 = 16 * (warp % nks) + g;  // position within the tile (key1 = key0 + 8)
  const uint32_t k_row0 = uint32_t(h * Tp + key0) * kRowBytes + 32 * c;
  const uint32_t k_row1 = k_row0 + 8 * kRowBytes;
  const uint32_t cs_row0 = uint32_t(key0) * kCsRow + kCsLane * c;
  const uint32_t cs_row1 = cs_row0 + 8 * kCsRow;

  // B fragments: b[nt][s][0..1] = q[row 8nt+g][dims of k-step s, slots c and c+4]
  uint32_t bq[kNT][16][2];
  {
    const T* qg = static_cast<const T*>(a.q);
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt) {
      const int r = 8 * nt + g;
      if (r < R) {
        const T* qr = qg + int64_t(b) * a.q_sb + int64_t(h * a.G + r / a.sq_n) * a.q_sh +
                      int64_t(a.s0 + r % a.sq_n) * a.q_ss;
#pragma unroll
        for (int s = 0; s < 16; ++s) {
          const int d = (s < 8) ? 16 * c + 2 * s : 64 + 16 * c + 2 * (s - 8);
          bq[nt][s][0] = __float_as_uint(to_f32(qr[d]));
          bq[nt][s][1] = __float_as_uint(to_f32(qr[d + 1]));
        }
      } else {
#pragma unroll
        for (int s = 0; s < 16; ++s) bq[nt][s][0] = bq[nt][s][1] = 0u;
      }
    }
  }
  // output rows of this lane: query rows 2c, 2c+1 of each n-tile
  float* out_row[kNT][2];
  int64_t vis[kNT][2];
  bool wr[kNT][2];
#pragma unroll
  for (int nt = 0; nt < kNT; ++nt) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int r = 8 * nt + 2 * c + e;
      wr[nt][e] = r < R;
      const int rr = min(r, R - 1);
      const int s_abs = a.s0 + rr % a.sq_n;
      out_row[nt][e] =
          a.scores + ((int64_t(b) * a.Hq + h * a.G + rr / a.sq_n) * a.Sq + s_abs) * a.ld;
      vis[nt][e] = a.causal ? a.causal_offset + s_abs : INT64_MAX;
    }
  }
  __syncthreads();

  const int kb_coord = (a.B > 1 && a.k_sb != 0) ? b : 0;
  auto issue = [&](int t, int s) {
    const uint64_t pol = l2_policy_evict_first();
    mbar_arrive_expect_tx(&tail->full[s], stage_bytes);
    tma_load_4d(stages + s * stage_bytes, &kmap, 0, t * Tp, 0, kb_coord, &tail->full[s], pol);
  };
  if (tid == 0) {
    for (int k = 0; k < kStages - 1 && t_begin + k < t_end; ++k) issue(t_begin + k, k);
  }

  const uint32_t smem_base = smem_u32(smem);
  const uint32_t cs_base = smem_u32(cs_tab);
  int it = 0;
  for (int t = t_begin; t < t_end; ++t, ++it) {
    const int p0 = t * Tp;
    const uint32_t cs_buf = cs_base + (it & 1) * Tp * kCsRow;
    if (kRope) {
      for (int idx = tid; idx < Tp * 32; idx += kThreads) {
        const int p = idx >> 5, qc = idx & 31;  // pairs 2qc, 2qc+1: lane block qc/8, chunk qc%8
        const float pf = static_cast<float>(a.pos_offset + p0 + p);
        float4 v;  // (cos f0, cos f1, sin f0, sin f1)
        rope_sincos_fast(__fmul_rn(pf, tail->inv_freq[2 * qc]), v.z, v.x);
        rope_sincos_fast(__fmul_rn(pf, tail->inv_freq[2 * qc + 1]), v.w, v.y);
        constexpr float kTruncScale = 1.0f + 0x1.0p-11f;  // see the precision note
        v.x *= kTruncScale;
        v.y *= kTruncScale;
        v.z *= kTruncScale;
        v.w *= kTruncScale;
        const uint32_t addr = cs_buf + p * kCsRow + kCsLane * (qc >> 3) + 16 * (qc & 7);
        asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "f"(v.x), "f"(v.y),
                     "f"(v.z), "f"(v.w)
                     : "memory");
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

    // rotated keys: kr[key][k-step] as (slot c, slot c+4) pairs
    float2 kr[2][16];
    const uint32_t st = smem_base + s * stage_bytes;
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      const uint32_t krow = st + (kk ? k_row1 : k_row0);
      const uint4 w0 = lds128_u32(krow), w1 = lds128_u32(krow + 16);
      const uint4 w2 = lds128_u32(krow + 128), w3 = lds128_u32(krow + 144);
      float2 lo[8], hi[8];  // dims 16c + 2i, +1 (and +64)
      unpack8<T>(w0, lo);
      unpack8<T>(w1, lo + 4);
      unpack8<T>(w2, hi);
      unpack8<T>(w3, hi + 4);
      if (kRope) {
        const uint32_t csr = cs_buf + (kk ? cs_row1 : cs_row0);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 cs = lds128f_u32(csr + 16 * i);  // pairs 16c+2i, 16c+2i+1
          const float2 cc = make_float2(cs.x, cs.y), ss = make_float2(cs.z, cs.w);
          const float2 ns = make_float2(-cs.z, -cs.w);
          kr[kk][i] = __ffma2_rn(hi[i], ss, __fmul2_rn(lo[i], cc));
          kr[kk][8 + i] = __ffma2_rn(lo[i], ns, __fmul2_rn(hi[i], cc));
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          kr[kk][i] = lo[i];
          kr[kk][8 + i] = hi[i];
        }
      }
    }
    float acc[kNT][2][4];
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
      for (int ch = 0; ch < 2; ++ch)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[nt][ch][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 16; ++ks) {
      const uint32_t a0 = __float_as_uint(kr[0][ks].x), a1 = __float_as_uint(kr[1][ks].x);
      const uint32_t a2 = __float_as_uint(kr[0][ks].y), a3 = __float_as_uint(kr[1][ks].y);
#pragma unroll
      for (int nt = 0; nt < kNT; ++nt)
        mma_tf32(acc[nt][ks & 1], a0, a1, a2, a3, bq[nt][ks][0], bq[nt][ks][1]);
    }
    // acc[nt][.][0..1]: key0, rows 2c, 2c+1; [2..3]: key1
    const int pos0 = p0 + key0, pos1 = pos0 + 8;
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        if (!wr[nt][e]) continue;
        const float v0 = acc[nt][0][e] + acc[nt][1][e];
        const float v1 = acc[nt][0][2 + e] + acc[nt][1][2 + e];
        if (pos0 < a.Sk) out_row[nt][e][pos0] = int64_t(pos0) > vis[nt][e] ? -INFINITY : v0;
        if (pos1 < a.Sk) out_row[nt][e][pos1] = int64_t(pos1) > vis[nt][e] ? -INFINITY : v1;
      }
    }
  }
}

size_t mma_smem_bytes(int Hkv, int Tp) {
  return size_t(kStages) * Hkv * Tp * kRowBytes + size_t(2) * Tp * kCsRow + sizeof(MmaTail);
}

template <typename T, bool kRope, int kNT>
cudaError_t launch_mma(const DecodeArgs& a, int num_sms, cudaStream_t stream) {
  const int Tp = 128 / a.Hkv;
  const size_t smem = mma_smem_bytes(a.Hkv, Tp);
  auto kern = decode_mma_kernel<T, kRope, kNT>;
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

template <typename T, bool kRope>
cudaError_t launch_mma_nt(const DecodeArgs& a, int num_sms, cudaStream_t stream) {
  const int R = a.G * a.sq_n;
  return R <= 8 ? launch_mma<T, kRope, 1>(a, num_sms, stream)
                : launch_mma<T, kRope, 2>(a, num_sms, stream);
}

}  // namespace

bool decode_mma_supported(const DecodeArgs& a) {
  const int R = a.G * a.sq_n;
  const int H = a.Hkv;
  return R <= 16 && (H == 2 || H == 4 || H == 8) && mma_smem_bytes(H, 128 / H) <= 227 * 1024;
}

cudaError_t launch_decode_scores_mma(const DecodeArgs& a, int dtype, int num_sms,
                                     cudaStream_t stream) {
  const bool rope = a.inv_freq != nullptr;
  if (dtype == kBF16)
    return rope ? launch_mma_nt<__nv_bfloat16, true>(a, num_sms, stream)
                : launch_mma_nt<__nv_bfloat16, false>(a, num_sms, stream);
  return rope ? launch_mma_nt<__half, true>(a, num_sms, stream)
              : launch_mma_nt<__half, false>(a, num_sms, stream);
}

}  // namespace prism
