// Decode-shaped scorer: q·K^T for a handful of query rows per KV head, with the
// inverse RoPE rotation of the cached keys fused into the key load.
//
// Reference path restated here (eval_harness/attention_methods):
//   ReAttentionMethod._unrotate_keys   reattention.py:743-793
//   undo_rotary_pos_emb / build_cos_sin _method_base.py:336-381
//   ReAttentionMethod._dense_topk       reattention.py:486-498  (einsum part)
//   GQA mapping kv_head = q_head // (Hq / Hkv), as _repeat_kv reattention.py:158-164
//
// Design (B200): the kernel is HBM-bound (256 B of K per key and KV head, ~770
// FLOP). One persistent CTA per SM streams key tiles of 128 positions x one KV
// head (32 KB, contiguous in HBM) through a 4-deep shared-memory ring with the
// TMA bulk-copy engine (cp.async.bulk + mbarrier, one producer warp). The
// eight consumer warps own 2 positions x 32 dims per thread: the RoPE cos/sin of
// those (position, frequency) pairs are computed once per tile and reused for
// every KV head and batch row; the un-rotated key stays in fp32 registers and is
// dotted against the fp32 query rows (resident in shared memory) of its GQA
// group. Scores go to an fp32 workspace that stays in L2 (keys are loaded with
// an evict-first policy) for the selection pass.
#include "common.cuh"
#include "kernels.h"
#include "rope_sincos.cuh"

namespace prism {
namespace {

constexpr int kT = 128;  // key positions per stage
constexpr int kStages = 4;
constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;  // + one producer warp
constexpr int kRC = 4;                     // query rows per register chunk
constexpr size_t kStageBytes = size_t(kT) * kRowBytes;

struct __align__(16) DecodeSmemTail {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  float inv_freq[64];
};

size_t decode_smem_bytes(int rows) {
  return kStages * kStageBytes + size_t(rows) * kHeadDim * sizeof(float) +
         sizeof(DecodeSmemTail);
}

template <typename T, bool kRope>
__global__ void __launch_bounds__(kThreads, 1) decode_scores_kernel(const DecodeArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* stages = smem;
  const int R = a.G * a.sq_n;  // query rows per KV-head group
  const int rows = a.Hkv * R;  // == Hq * sq_n rows resident for this batch
  float* q_s = reinterpret_cast<float*>(smem + kStages * kStageBytes);
  DecodeSmemTail* tail = reinterpret_cast<DecodeSmemTail*>(q_s + size_t(rows) * kHeadDim);

  const int tid = threadIdx.x;
  const int b = blockIdx.y;
  const int t_begin = static_cast<int>(int64_t(blockIdx.x) * a.ntiles / gridDim.x);
  const int t_end = static_cast<int>(int64_t(blockIdx.x + 1) * a.ntiles / gridDim.x);

  asm volatile("griddepcontrol.launch_dependents;");
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&tail->full[s], 1);
      mbar_init(&tail->empty[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  // q rows of this batch, fp32, laid out [kv head][row in group][dim].
  const T* qg = static_cast<const T*>(a.q);
  for (int e = tid; e < rows * kHeadDim; e += kThreads) {
    const int row = e / kHeadDim, d = e % kHeadDim;
    const int hk = row / R, r = row % R;
    const int gi = r / a.sq_n, sl = r % a.sq_n;
    const int hq = hk * a.G + gi;
    q_s[e] = to_f32(qg[int64_t(b) * a.q_sb + int64_t(hq) * a.q_sh +
                       int64_t(a.s0 + sl) * a.q_ss + d]);
  }
  if (kRope) {
    for (int i = tid; i < kHeadDim / 2; i += kThreads) tail->inv_freq[i] = a.inv_freq[i];
  }
  __syncthreads();

  const int warp = tid >> 5, lane = tid & 31;
  if (warp == kConsumerWarps) {
    // ---------------- producer warp: one lane issues all bulk copies ----------
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      const uint8_t* kbase =
          static_cast<const uint8_t*>(a.k) + int64_t(b) * a.k_sb * int64_t(sizeof(T));
      int it = 0;
      for (int t = t_begin; t < t_end; ++t) {
        const int p0 = t * kT;
        const int nvalid = min(kT, a.Sk - p0);
        const uint32_t bytes = uint32_t(nvalid) * kRowBytes;
        for (int hk = 0; hk < a.Hkv; ++hk, ++it) {
          const int s = it % kStages;
          if (it >= kStages) {
            if (!mbar_wait_bounded(&tail->empty[s], ((it / kStages) - 1) & 1)) {
              set_status(a.status, kStatusTimeout);
              return;
            }
          }
          mbar_arrive_expect_tx(&tail->full[s], bytes);
          bulk_g2s(stages + s * kStageBytes,
                   kbase + (int64_t(hk) * a.k_sh + int64_t(p0) * kHeadDim) * int64_t(sizeof(T)),
                   bytes, &tail->full[s], pol);
        }
      }
    }
    return;
  }

  // ---------------- consumer warps ----------------------------------------
  const int quad = tid >> 2;  // 0..63: positions quad and quad + 64 of a tile
  const int j = tid & 3;      // dims [16j, 16j+16) and [64+16j, 64+16j+16)
  float cs[2][16], sn[2][16];
  int it = 0;
  for (int t = t_begin; t < t_end; ++t) {
    const int p0 = t * kT;
    if (kRope) {
#pragma unroll
      for (int pp = 0; pp < 2; ++pp) {
        const float pf = static_cast<float>(a.pos_offset + p0 + quad + 64 * pp);
#pragma unroll
        for (int u = 0; u < 16; ++u)
          rope_sincos(__fmul_rn(pf, tail->inv_freq[16 * j + u]), sn[pp][u], cs[pp][u]);
      }
    }
    for (int hk = 0; hk < a.Hkv; ++hk, ++it) {
      const int s = it % kStages;
      // warp-uniform outcome: a timeout in any lane retires the whole warp
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&tail->full[s], (it / kStages) & 1))) {
        set_status(a.status, kStatusTimeout);
        return;
      }
      const uint8_t* st = stages + s * kStageBytes;
      float kr[2][32];
#pragma unroll
      for (int pp = 0; pp < 2; ++pp) {
        const uint8_t* rowp = st + (quad + 64 * pp) * kRowBytes;
        uint4 w[4];
        w[0] = lds128(rowp + 32 * j);
        w[1] = lds128(rowp + 32 * j + 16);
        w[2] = lds128(rowp + 128 + 32 * j);
        w[3] = lds128(rowp + 128 + 32 * j + 16);
        float lo[16], hi[16];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          Unpack<T>::run(w[c].x, lo[8 * c + 0], lo[8 * c + 1]);
          Unpack<T>::run(w[c].y, lo[8 * c + 2], lo[8 * c + 3]);
          Unpack<T>::run(w[c].z, lo[8 * c + 4], lo[8 * c + 5]);
          Unpack<T>::run(w[c].w, lo[8 * c + 6], lo[8 * c + 7]);
          Unpack<T>::run(w[2 + c].x, hi[8 * c + 0], hi[8 * c + 1]);
          Unpack<T>::run(w[2 + c].y, hi[8 * c + 2], hi[8 * c + 3]);
          Unpack<T>::run(w[2 + c].z, hi[8 * c + 4], hi[8 * c + 5]);
          Unpack<T>::run(w[2 + c].w, hi[8 * c + 6], hi[8 * c + 7]);
        }
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          if (kRope) {
            kr[pp][u] = fmaf(hi[u], sn[pp][u], lo[u] * cs[pp][u]);
            kr[pp][16 + u] = fmaf(-lo[u], sn[pp][u], hi[u] * cs[pp][u]);
          } else {
            kr[pp][u] = lo[u];
            kr[pp][16 + u] = hi[u];
          }
        }
      }
      const float* qgrp = q_s + size_t(hk) * R * kHeadDim;
      for (int r0 = 0; r0 < R; r0 += kRC) {
        float v[8];  // v[rr*2 + pp]
#pragma unroll
        for (int rr = 0; rr < kRC; ++rr) {
          const int r = min(r0 + rr, R - 1);
          const float* qr = qgrp + r * kHeadDim;
          float qv[32];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const float4 x = *reinterpret_cast<const float4*>(qr + 16 * j + 4 * c);
            const float4 y = *reinterpret_cast<const float4*>(qr + 64 + 16 * j + 4 * c);
            qv[4 * c + 0] = x.x; qv[4 * c + 1] = x.y; qv[4 * c + 2] = x.z; qv[4 * c + 3] = x.w;
            qv[16 + 4 * c + 0] = y.x; qv[16 + 4 * c + 1] = y.y;
            qv[16 + 4 * c + 2] = y.z; qv[16 + 4 * c + 3] = y.w;
          }
#pragma unroll
          for (int pp = 0; pp < 2; ++pp) {
            float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
            for (int u = 0; u < 32; u += 2) {
              acc0 = fmaf(qv[u], kr[pp][u], acc0);
              acc1 = fmaf(qv[u + 1], kr[pp][u + 1], acc1);
            }
            v[rr * 2 + pp] = acc0 + acc1;
          }
        }
        // Transposed reduction across the 4 lanes of the quad: afterwards lane j
        // holds the full sums of row r0 + j for both positions.
        const bool b1 = (j & 2) != 0, b0 = (j & 1) != 0;
        float u4[4];
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const float send = b1 ? v[m] : v[m + 4];
          const float keep = b1 ? v[m + 4] : v[m];
          u4[m] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
        }
        float w2[2];
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          const float send = b0 ? u4[m] : u4[m + 2];
          const float keep = b0 ? u4[m + 2] : u4[m];
          w2[m] = keep + __shfl_xor_sync(0xffffffffu, send, 1);
        }
        const int r = r0 + j;
        if (r < R) {
          const int gi = r / a.sq_n, sl = r % a.sq_n;
          const int s_abs = a.s0 + sl;
          const int64_t row = (int64_t(b) * a.Hq + hk * a.G + gi) * a.Sq + s_abs;
          float* out = a.scores + row * a.ld;
#pragma unroll
          for (int pp = 0; pp < 2; ++pp) {
            const int p = p0 + quad + 64 * pp;
            if (p < a.Sk) {
              float val = w2[pp];
              if (a.causal && int64_t(p) > a.causal_offset + s_abs) val = -INFINITY;
              out[p] = val;
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&tail->empty[s]);
    }
  }
}

template <typename T, bool kRope>
cudaError_t launch_impl(const DecodeArgs& a, int num_sms, cudaStream_t stream) {
  const int rows = a.Hq * a.sq_n;
  const size_t smem = decode_smem_bytes(rows);
  auto kern = decode_scores_kernel<T, kRope>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int ctas = num_sms;
  if (a.B > 1) ctas = (num_sms + a.B - 1) / a.B;
  ctas = max(1, min(ctas, a.ntiles));
  dim3 grid(ctas, a.B);
  kern<<<grid, kThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_decode_scores(const DecodeArgs& a, int dtype, int num_sms,
                                 cudaStream_t stream) {
  const bool rope = a.inv_freq != nullptr;
  if (dtype == kBF16)
    return rope ? launch_impl<__nv_bfloat16, true>(a, num_sms, stream)
                : launch_impl<__nv_bfloat16, false>(a, num_sms, stream);
  return rope ? launch_impl<__half, true>(a, num_sms, stream)
              : launch_impl<__half, false>(a, num_sms, stream);
}

}  // namespace prism
