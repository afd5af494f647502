// Scorer for many query rows per KV head (up to 256 / Hkv, e.g. 8 questions x 7
// heads of a GQA group sharing one context): queries are the MMA's M dimension.
//
// Reference path: ReAttentionMethod._unrotate_keys + _dense_topk's einsum
// (eval_harness/attention_methods/reattention.py:743-793, 486-498), GQA mapping
// kv head = q head / (Hq / Hkv).
//
// One mma.sync m16n8k8 TF32 tile = 16 query rows x 8 keys of one KV head, k-step
// of 8 dims. Lane (g, c) supplies key g's dims (16c + 2s, 16c + 2s + 1) for k-step
// s < 8 and the same dims + 64 for k-step 8 + s: its keys' rotation pairs
// [16c, 16c + 16) of both halves, so the inverse RoPE rotation stays inside the
// lane and the rotated values are the B fragments directly. The query rows'
// A fragments of a warp's (head, m-tile) pairs live in registers for the whole
// kernel (64 registers per m-tile).
//
// Layout: a stage is Tp = 128 / Hkv positions x all KV heads (one tiled TMA
// copy, 32 KB) in a 4-deep ring; cos/sin of the stage's positions are computed
// once into a double-buffered shared table (one angle per (position, frequency),
// shared by all heads and m-tiles). 8 warps: warp w takes head w / (8 / Hkv) and
// up to kMT m-tiles of it, and loops over the stage's 8-key n-tiles of that head.
// Thread 0 waits for each stage; the block barrier then publishes the stage and
// the cos/sin table, and only after it is the stage of the previous iteration
// refilled.
//
// Modes (the epilogue's work):
//   kWScores  the fp32 score matrix [rows, ld] (masked keys -inf);
//   kWSample  the scores of every tstride-th stage only (a threshold sample:
//             Tp consecutive positions of every tstride * Tp), written compactly
//             to [rows, ld] with sample column = sampled stage * Tp + offset;
//   kWCand    no scores: every visible key scoring at or above its row's
//             threshold thr[row] (NaN included) is appended, packed as
//             (fp32 score bits << 32) | ~key, to the row's candidate list
//             [rows, cap] through a per-row counter (counts[2 row]; the count
//             may exceed cap, which the selection then recomputes exactly).
//
// Precision: as in the other tensor-core scorers, cos/sin are scaled by
// (1 + 2^-11) so that the operand truncation of TF32 lands within 2^-11 of the
// rotated key; queries (bf16/fp16) are exact in TF32, accumulation is fp32.
#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "rope_sincos.cuh"
#include "tensor_map.h"

namespace prism {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kStages = 4;             // key ring depth (3 in the candidate mode)
constexpr int kCandBuf = 16;           // candidate mode: entries per row staged in shared memory
constexpr int kCandFlush = 4;          // candidate mode: stages between flushes
constexpr int kMaxLocalRows = 256;     // Hkv * rows per KV head
constexpr int kCsRow = 576;   // bytes per position in the cos/sin table
constexpr int kCsLane = 144;  // bytes between consecutive lanes' 128-byte blocks
constexpr float kTruncScale = 1.0f + 0x1.0p-11f;

enum WideMode : int { kWScores = 0, kWSample = 1, kWCand = 2 };

struct WideExtra {
  int tstride;            // kWSample: every tstride-th stage
  const float* thr;       // kWCand: per-row thresholds
  uint32_t* counts;       // kWCand: [rows, 2] (front list count, 0)
  uint64_t* cand;         // kWCand: [rows, cap]
  int64_t cap;
};

struct __align__(16) WideTail {
  uint64_t full[kStages];
  float inv_freq[64];
  int abort;
};

__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ int dim_of(int s, int c) {
  return s < 8 ? 16 * c + 2 * s : 64 + 16 * c + 2 * (s - 8);
}

__host__ __device__ constexpr int wide_stages(int mode) { return mode == 2 ? 3 : kStages; }

template <typename T, bool kRope, int kMT, int kMode>
__global__ void __launch_bounds__(kThreads, 1)
    decode_wide_kernel(const __grid_constant__ CUtensorMap kmap, const DecodeArgs a, int Tp,
                       const WideExtra x) {
  constexpr int kStages = wide_stages(kMode);
  extern __shared__ __align__(128) uint8_t smem[];
  const int Hkv = a.Hkv;
  const int R = a.G * a.sq_n;
  const int M = (R + 15) / 16;                   // m-tiles per head
  const int wph = kWarps / Hkv;                  // warps per head
  const uint32_t stage_bytes = uint32_t(Hkv) * Tp * kRowBytes;
  uint8_t* stages = smem;
  uint8_t* cs_tab = smem + kStages * stage_bytes;  // [2][Tp][kCsRow]
  WideTail* tail = reinterpret_cast<WideTail*>(cs_tab + 2 * Tp * kCsRow);
  // candidate mode: per (KV head, row) a small staging list in shared memory,
  // flushed to the row's global list every kCandFlush stages with one atomic
  uint32_t* ccount = reinterpret_cast<uint32_t*>(tail + 1);          // [kMaxLocalRows]
  uint64_t* cbuf = reinterpret_cast<uint64_t*>(ccount + kMaxLocalRows);  // [kMaxLocalRows][kCandBuf]

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int h = warp / wph;                      // this warp's KV head
  const int mt0 = (warp % wph) * kMT;            // its first m-tile
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
  if (kMode == kWCand) {
    for (int i = tid; i < kMaxLocalRows; i += kThreads) ccount[i] = 0u;
  }
  // score row of local row lr = h * R + r (KV head h, row r of its query group)
  auto score_row = [&](int lr) -> int64_t {
    const int hh = lr / R, r = lr - hh * R;
    return (int64_t(b) * a.Hq + hh * a.G + r / a.sq_n) * a.Sq + a.s0 + r % a.sq_n;
  };
  // moves every staged candidate to its row's global list (all threads; the
  // caller brackets it with block barriers)
  auto flush = [&]() {
    for (int lr = tid; lr < Hkv * R; lr += kThreads) {
      const uint32_t n = min(ccount[lr], uint32_t(kCandBuf));
      if (n == 0) continue;
      const int64_t srow = score_row(lr);
      const uint32_t base = atomicAdd(&x.counts[2 * srow], n);
      for (uint32_t e = 0; e < n; ++e)
        if (base + e < uint64_t(x.cap)) x.cand[srow * x.cap + base + e] = cbuf[lr * kCandBuf + e];
      ccount[lr] = 0u;
    }
  };

  // A fragments of this warp's m-tiles: rows 16 mt + g (+ 8), dims of k-step s
  // at columns c (a0, a1) and c + 4 (a2, a3)
  uint32_t aq[kMT][16][4];
  const T* qg = static_cast<const T*>(a.q);
#pragma unroll
  for (int j = 0; j < kMT; ++j) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int r = 16 * (mt0 + j) + g + 8 * half;
      const bool live = mt0 + j < M && r < R;
      const T* qr = qg + int64_t(b) * a.q_sb + int64_t(h * a.G + (live ? r : 0) / a.sq_n) * a.q_sh +
                    int64_t(a.s0 + (live ? r : 0) % a.sq_n) * a.q_ss;
      // dims 16c + 2s, +1 (k-step s < 8) and 64 + 16c + 2(s - 8), +1 (s >= 8): two
      // runs of 16 elements, read as 16-byte words when the row is aligned
      if (live && (reinterpret_cast<uintptr_t>(qr) & 15u) == 0) {
        uint4 w[4];
        w[0] = __ldg(reinterpret_cast<const uint4*>(qr + 16 * c));
        w[1] = __ldg(reinterpret_cast<const uint4*>(qr + 16 * c + 8));
        w[2] = __ldg(reinterpret_cast<const uint4*>(qr + 64 + 16 * c));
        w[3] = __ldg(reinterpret_cast<const uint4*>(qr + 64 + 16 * c + 8));
        const uint32_t ws[16] = {w[0].x, w[0].y, w[0].z, w[0].w, w[1].x, w[1].y, w[1].z, w[1].w,
                                 w[2].x, w[2].y, w[2].z, w[2].w, w[3].x, w[3].y, w[3].z, w[3].w};
#pragma unroll
        for (int s = 0; s < 16; ++s) {
          float lo, hi;
          Unpack<T>::run(ws[s], lo, hi);
          aq[j][s][half] = __float_as_uint(lo);
          aq[j][s][2 + half] = __float_as_uint(hi);
        }
      } else {
#pragma unroll
        for (int s = 0; s < 16; ++s) {
          const int d = dim_of(s, c);
          aq[j][s][half] = live ? __float_as_uint(to_f32(qr[d])) : 0u;
          aq[j][s][2 + half] = live ? __float_as_uint(to_f32(qr[d + 1])) : 0u;
        }
      }
    }
  }
  // output rows of this lane: 16 mt + g and + 8 of each m-tile (score row index;
  // row_off = the row's offset in the score matrix, thr_row its threshold)
  int64_t row_off[kMT][2];
  int64_t vis[kMT][2];
  bool wr[kMT][2];
  float thr_row[kMT][2];
#pragma unroll
  for (int j = 0; j < kMT; ++j) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int r = 16 * (mt0 + j) + g + 8 * half;
      wr[j][half] = mt0 + j < M && r < R;
      const int rr = r < R ? r : R - 1;
      const int s_abs = a.s0 + rr % a.sq_n;
      const int64_t srow = (int64_t(b) * a.Hq + h * a.G + rr / a.sq_n) * a.Sq + s_abs;
      row_off[j][half] = kMode == kWCand ? srow : srow * a.ld;
      vis[j][half] = a.causal ? a.causal_offset + s_abs : INT64_MAX;
      thr_row[j][half] = kMode == kWCand && wr[j][half] ? x.thr[srow] : 0.f;
    }
  }
  __syncthreads();

  const int kb_coord = (a.B > 1 && a.k_sb != 0) ? b : 0;
  // stage t of the loop holds keys of tile t * tstride (kWSample) or t
  const int tstep = kMode == kWSample ? x.tstride : 1;
  auto issue = [&](int t, int s) {
    const uint64_t pol = l2_policy_evict_first();
    mbar_arrive_expect_tx(&tail->full[s], stage_bytes);
    tma_load_4d(stages + s * stage_bytes, &kmap, 0, t * tstep * Tp, 0, kb_coord, &tail->full[s], pol);
  };
  if (tid == 0) {
    for (int k = 0; k < kStages - 1 && t_begin + k < t_end; ++k) issue(t_begin + k, k);
  }

  const uint32_t smem_base = smem_u32(smem);
  const uint32_t cs_base = smem_u32(cs_tab);
  const bool active = mt0 < M;
  int it = 0;
  for (int t = t_begin; t < t_end; ++t, ++it) {
    const int p0 = t * tstep * Tp;  // the stage's first key position
    const int c0 = t * Tp;          // kWSample: its first sample column
    const uint32_t cs_buf = cs_base + (it & 1) * Tp * kCsRow;
    if (kRope) {
      for (int idx = tid; idx < Tp * 32; idx += kThreads) {
        const int p = idx >> 5, qc = idx & 31;  // pairs 2qc, 2qc+1: lane block qc/8, chunk qc%8
        const float pf = static_cast<float>(a.pos_offset + p0 + p);
        float4 v;  // (cos f0, cos f1, sin f0, sin f1)
        rope_sincos_fast(__fmul_rn(pf, tail->inv_freq[2 * qc]), v.z, v.x);
        rope_sincos_fast(__fmul_rn(pf, tail->inv_freq[2 * qc + 1]), v.w, v.y);
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
    __syncthreads();  // stage t and its cos/sin are ready; every warp is past stage t-1
    if (tail->abort) return;
    if (tid == 0 && t + kStages - 1 < t_end) issue(t + kStages - 1, (it + kStages - 1) % kStages);
    if (kMode == kWCand && it > 0 && it % kCandFlush == 0) {
      flush();
      __syncthreads();  // the staging lists are empty again
    }
    if (!active) continue;

    const uint32_t st = smem_base + s * stage_bytes;
    for (int n0 = 0; n0 < Tp; n0 += 8) {
      const int pl = n0 + g;  // this lane's key within the stage
      const uint32_t krow = st + uint32_t(h * Tp + pl) * kRowBytes + 32 * c;
      const uint4 w0 = lds128_u32(krow), w1 = lds128_u32(krow + 16);
      const uint4 w2 = lds128_u32(krow + 128), w3 = lds128_u32(krow + 144);
      const uint32_t kwl[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      const uint32_t kwh[8] = {w2.x, w2.y, w2.z, w2.w, w3.x, w3.y, w3.z, w3.w};
      float2 kr[16];
      const uint32_t csr = cs_buf + uint32_t(pl) * kCsRow + kCsLane * c;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float2 lo, hi;
        Unpack<T>::run(kwl[i], lo.x, lo.y);
        Unpack<T>::run(kwh[i], hi.x, hi.y);
        if (kRope) {
          const float4 cs = lds128f_u32(csr + 16 * i);  // pairs 16c+2i, 16c+2i+1
          const float2 cc = make_float2(cs.x, cs.y), ss = make_float2(cs.z, cs.w);
          const float2 ns = make_float2(-cs.z, -cs.w);
          kr[i] = __ffma2_rn(hi, ss, __fmul2_rn(lo, cc));
          kr[8 + i] = __ffma2_rn(lo, ns, __fmul2_rn(hi, cc));
        } else {
          kr[i] = lo;
          kr[8 + i] = hi;
        }
      }
      // two accumulators per m-tile (k-steps 0-7 and 8-15), so that each warp keeps
      // 2 kMT independent MMA chains in flight, summed at the end
      float acc[kMT][4], acc2[kMT][4];
#pragma unroll
      for (int j = 0; j < kMT; ++j) {
        acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
        acc2[j][0] = acc2[j][1] = acc2[j][2] = acc2[j][3] = 0.f;
      }
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
        for (int j = 0; j < kMT; ++j) {
          mma_tf32(acc[j], aq[j][ks], __float_as_uint(kr[ks].x), __float_as_uint(kr[ks].y));
          mma_tf32(acc2[j], aq[j][8 + ks], __float_as_uint(kr[8 + ks].x), __float_as_uint(kr[8 + ks].y));
        }
      }
#pragma unroll
      for (int j = 0; j < kMT; ++j) {
        acc[j][0] += acc2[j][0];
        acc[j][1] += acc2[j][1];
        acc[j][2] += acc2[j][2];
        acc[j][3] += acc2[j][3];
      }
      // acc[j]: (row g, keys 2c, 2c+1), (row g+8, keys 2c, 2c+1)
      const int pos = p0 + n0 + 2 * c;
#pragma unroll
      for (int j = 0; j < kMT; ++j) {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          if (!wr[j][half]) continue;
          if (kMode == kWCand) {
            // visible keys at or above the row's threshold (!(v < thr): NaN too)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int p = pos + e;
              const float v = acc[j][2 * half + e];
              if (p < a.Sk && int64_t(p) <= vis[j][half] && !(v < thr_row[j][half])) {
                const uint64_t pk = (uint64_t(__float_as_uint(v)) << 32) | uint64_t(~uint32_t(p));
                const int lr = h * R + 16 * (mt0 + j) + g + 8 * half;
                const uint32_t slot = atomicAdd(&ccount[lr], 1u);
                if (slot < uint32_t(kCandBuf)) {
                  cbuf[lr * kCandBuf + slot] = pk;
                } else {  // the staging list is full: straight to the row's list
                  const int64_t srow = row_off[j][half];
                  const uint32_t gs = atomicAdd(&x.counts[2 * srow], 1u);
                  if (gs < uint64_t(x.cap)) x.cand[srow * x.cap + gs] = pk;
                }
              }
            }
            continue;
          }
          const float v0 = int64_t(pos) > vis[j][half] ? -INFINITY : acc[j][2 * half];
          const float v1 = int64_t(pos + 1) > vis[j][half] ? -INFINITY : acc[j][2 * half + 1];
          if (kMode == kWSample) {
            // every sample column of the stage is written, beyond Sk too (as -inf:
            // the threshold kernel skips columns past the end)
            float* o = a.scores + row_off[j][half] + c0 + n0 + 2 * c;
            *reinterpret_cast<float2*>(o) = make_float2(pos < a.Sk ? v0 : -INFINITY,
                                                        pos + 1 < a.Sk ? v1 : -INFINITY);
            continue;
          }
          float* o = a.scores + row_off[j][half];
          if (pos + 1 < a.Sk) {
            *reinterpret_cast<float2*>(o + pos) = make_float2(v0, v1);
          } else if (pos < a.Sk) {
            o[pos] = v0;
          }
        }
      }
    }
  }
  if (kMode == kWCand) {
    __syncthreads();  // every warp is done with its last stage
    flush();
  }
}

size_t wide_smem_bytes(int Hkv, int Tp, int mode = kWScores) {
  return size_t(wide_stages(mode)) * Hkv * Tp * kRowBytes + size_t(2) * Tp * kCsRow + sizeof(WideTail) +
         (mode == kWCand ? size_t(kMaxLocalRows) * (4 + 8 * kCandBuf) : 0);
}

template <typename T, bool kRope, int kMT, int kMode>
cudaError_t launch_wide(const DecodeArgs& a, int num_sms, const WideExtra& x, cudaStream_t stream) {
  const int Tp = 128 / a.Hkv;
  const size_t smem = wide_smem_bytes(a.Hkv, Tp, kMode);
  auto kern = decode_wide_kernel<T, kRope, kMT, kMode>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  CUtensorMap kmap;
  e = make_key_tensor_map(&kmap, a.k, std::is_same<T, __nv_bfloat16>::value ? kBF16 : kFP16, a.B,
                          a.Hkv, a.Sk, a.k_sb, a.k_sh, Tp);
  if (e != cudaSuccess) return e;
  DecodeArgs b = a;
  b.ntiles = (a.Sk + Tp - 1) / Tp;
  if (kMode == kWSample) b.ntiles = (b.ntiles + x.tstride - 1) / x.tstride;  // sampled stages
  int ctas = num_sms;
  if (a.B > 1) ctas = (num_sms + a.B - 1) / a.B;
  ctas = max(1, min(ctas, b.ntiles));
  kern<<<dim3(ctas, a.B), kThreads, smem, stream>>>(kmap, b, Tp, x);
  return cudaGetLastError();
}

template <typename T, bool kRope, int kMode>
cudaError_t launch_wide_mt(const DecodeArgs& a, int num_sms, const WideExtra& x, cudaStream_t stream) {
  const int M = (a.G * a.sq_n + 15) / 16;
  const int wph = kWarps / a.Hkv;
  return M <= wph ? launch_wide<T, kRope, 1, kMode>(a, num_sms, x, stream)
                  : launch_wide<T, kRope, 2, kMode>(a, num_sms, x, stream);
}

template <int kMode>
cudaError_t launch_wide_mode(const DecodeArgs& a, int dtype, int num_sms, const WideExtra& x,
                             cudaStream_t stream) {
  const bool rope = a.inv_freq != nullptr;
  if (dtype == kBF16)
    return rope ? launch_wide_mt<__nv_bfloat16, true, kMode>(a, num_sms, x, stream)
                : launch_wide_mt<__nv_bfloat16, false, kMode>(a, num_sms, x, stream);
  return rope ? launch_wide_mt<__half, true, kMode>(a, num_sms, x, stream)
              : launch_wide_mt<__half, false, kMode>(a, num_sms, x, stream);
}

}  // namespace

bool decode_wide_supported(const DecodeArgs& a) {
  const int H = a.Hkv;
  if (H != 2 && H != 4 && H != 8) return false;
  const int M = (a.G * a.sq_n + 15) / 16;
  const int wph = kWarps / H;
  return M <= 2 * wph && (reinterpret_cast<uintptr_t>(a.scores) & 7u) == 0 && a.ld % 2 == 0 &&
         wide_smem_bytes(H, 128 / H) <= 227 * 1024;
}

cudaError_t launch_decode_scores_wide(const DecodeArgs& a, int dtype, int num_sms,
                                      cudaStream_t stream) {
  return launch_wide_mode<kWScores>(a, dtype, num_sms, WideExtra{1, nullptr, nullptr, nullptr, 0}, stream);
}

int64_t wide_sample_cols(int Hkv, int64_t Sk) {
  const int64_t Tp = 128 / Hkv;
  const int64_t ntiles = (Sk + Tp - 1) / Tp;
  return (ntiles + kWideSampleStride - 1) / kWideSampleStride * Tp;
}

cudaError_t launch_wide_sample(const DecodeArgs& a, int dtype, int num_sms, cudaStream_t stream) {
  return launch_wide_mode<kWSample>(a, dtype, num_sms,
                                    WideExtra{kWideSampleStride, nullptr, nullptr, nullptr, 0}, stream);
}

cudaError_t launch_wide_candidates(const DecodeArgs& a, int dtype, const float* thr, uint32_t* counts,
                                   uint64_t* cand, int64_t cap, int num_sms, cudaStream_t stream) {
  return launch_wide_mode<kWCand>(a, dtype, num_sms, WideExtra{1, thr, counts, cand, cap}, stream);
}

}  // namespace prism
