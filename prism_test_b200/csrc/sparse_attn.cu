// Attention over the selected [global | recalled | local] view — the step after
// the recall selection in the exact method: ReAttentionExactMethod._chunk_attention
// gathers the view's keys and values from the raw (pre-RoPE) cache by absolute
// position, rotates keys and queries at their RoPE positions and attends
// (eval_harness/attention_methods/reattention_exact.py:453-508), with the eager
// path of _attend (:650-661): softmax(q k^T * scale) v in fp32, keys past a
// query's absolute position masked, fully masked rows giving zeros.
//
// sparse_attn_partial_kernel: a CTA takes up to kRB (4 or 8) query rows (g-major rows of
// one (batch, KV head)) and one split of the view; each of its 8 warps walks a
// contiguous share of the split's keys, 8 at a time (their rows all requested
// before the first is used): the key and value rows are gathered with one
// coalesced 8-byte load per lane (lane L holds dimensions 4L .. 4L+3), the
// key is rotated from the view's angle table (rope_table_kernel: (cos, sin) of
// every position and frequency; lanes L and L ^ 16 hold the two halves of a
// rotation pair), dotted with every query row (fp32, warp reduction), and folded
// into the row's online softmax (running max, sum and the unnormalised value
// accumulator). The warps' states are merged in shared memory and the CTA writes
// one partial (m, l, acc[128]) per row and split.
// sparse_attn_combine_kernel merges the splits of each row and writes the output.
// The partial and combine kernels are dependent launches: each starts while its
// predecessor drains and waits (griddepcontrol.wait) before reading its output.
#include "common.cuh"
#include "kernels.h"
#include "rope_sincos.cuh"

namespace prism {
namespace {

constexpr int kSaWarps = 8;

template <typename T>
__device__ __forceinline__ float4 load4(const T* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  float4 f;
  Unpack<T>::run(u.x, f.x, f.y);
  Unpack<T>::run(u.y, f.z, f.w);
  return f;
}

template <typename T>
__device__ __forceinline__ void store4(T* p, float4 f);
template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* p, float4 f) {
  __nv_bfloat162 a = __floats2bfloat162_rn(f.x, f.y), b = __floats2bfloat162_rn(f.z, f.w);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&a);
  u.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}
template <>
__device__ __forceinline__ void store4<__half>(__half* p, float4 f) {
  __half2 a = __floats2half2_rn(f.x, f.y), b = __floats2half2_rn(f.z, f.w);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&a);
  u.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}

// x[i] of a small register array with a lane-dependent i, by selects (no local memory)
template <int N, typename V>
__device__ __forceinline__ V pick(const V (&x)[N], int i) {
  V r = x[0];
#pragma unroll
  for (int k = 1; k < N; ++k) r = i == k ? x[k] : r;
  return r;
}
template <int N>
__device__ __forceinline__ int pu_at(const int (&x)[N], int i) { return pick<N, int>(x, i); }
template <int N>
__device__ __forceinline__ int64_t qabs_at(const int64_t (&x)[N], int i) { return pick<N, int64_t>(x, i); }

// RoPE of the lane's 4 dimensions from a table row of (cos, sin) per frequency
// (64 float2): lanes L < 16 hold x_i, lanes L + 16 hold x_{i+64}, i = 4 (L mod 16) + e.
__device__ __forceinline__ float4 rope4_table(float4 x, const float2* row, int lane) {
  const float4* t = reinterpret_cast<const float4*>(row + ((4 * lane) & 63));
  const float4 cs01 = t[0], cs23 = t[1];  // (c0, s0, c1, s1), (c2, s2, c3, s3)
  float4 p;  // partner half
  p.x = __shfl_xor_sync(0xffffffffu, x.x, 16);
  p.y = __shfl_xor_sync(0xffffffffu, x.y, 16);
  p.z = __shfl_xor_sync(0xffffffffu, x.z, 16);
  p.w = __shfl_xor_sync(0xffffffffu, x.w, 16);
  const float sg = (lane & 16) ? 1.f : -1.f;
  float4 o;
  o.x = fmaf(sg * p.x, cs01.y, x.x * cs01.x);
  o.y = fmaf(sg * p.y, cs01.w, x.y * cs01.z);
  o.z = fmaf(sg * p.z, cs23.y, x.z * cs23.x);
  o.w = fmaf(sg * p.w, cs23.w, x.w * cs23.z);
  return o;
}

__device__ __forceinline__ float dot4(float4 a, float4 b) {
  return fmaf(a.x, b.x, fmaf(a.y, b.y, fmaf(a.z, b.z, a.w * b.w)));
}

// kRB: query rows per CTA (4 for decode's GQA groups, 8 otherwise)
template <typename T, bool kRope, int kRB>
__global__ void __launch_bounds__(kSaWarps * 32, kRB == 4 ? 2 : 1)
    sparse_attn_partial_kernel(const SparseAttnArgs a) {
  __shared__ float s_m[kSaWarps][kRB], s_l[kSaWarps][kRB];
  __shared__ float4 s_acc[kSaWarps][kRB][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t R = int64_t(a.G) * a.Sq;  // query rows of a KV head
  const int nrb = int((R + kRB - 1) / kRB);
  const int rb = blockIdx.x % nrb;
  const int bh = blockIdx.x / nrb;
  const int b = bh / a.Hkv, h = bh - b * a.Hkv;
  const int split = blockIdx.y, nsplit = gridDim.y;
  const int64_t per = (a.nsel + nsplit - 1) / nsplit;
  const int64_t j0 = int64_t(split) * per;
  const int64_t j1 = j0 + per < a.nsel ? j0 + per : a.nsel;

  const int64_t r0 = int64_t(rb) * kRB;
  const int nrows = int(R - r0 < kRB ? R - r0 : kRB);

  // the queries (fp32, 4 dims per lane; with RoPE rotated and scaled by the
  // table kernel, read after the wait) and their absolute positions
  float4 q[kRB];
  int64_t qabs[kRB];
#pragma unroll
  for (int r = 0; r < kRB; ++r) {
    q[r] = make_float4(0.f, 0.f, 0.f, 0.f);
    qabs[r] = -1;
    if (r < nrows) {
      const int64_t rr = r0 + r, g = rr / a.Sq, s = rr - g * a.Sq;
      qabs[r] = a.q_pos[s];
      if (!kRope) {
        const T* qr = static_cast<const T*>(a.q) + int64_t(b) * a.q_sb +
                      (int64_t(h) * a.G + g) * a.q_sh + s * a.q_ss;
        q[r] = load4<T>(qr + 4 * lane);
        q[r].x *= a.scale;
        q[r].y *= a.scale;
        q[r].z *= a.scale;
        q[r].w *= a.scale;
      }
    }
  }
  // the angle table and the rotated queries (a dependent launch after
  // rope_table_kernel) are complete and visible after this; the combine kernel
  // may launch now
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
  if (kRope) {
#pragma unroll
    for (int r = 0; r < kRB; ++r) {
      if (r < nrows) {
        const int64_t rr = r0 + r, g = rr / a.Sq, s = rr - g * a.Sq;
        const int64_t orow = (int64_t(b) * a.Hq + int64_t(h) * a.G + g) * a.Sq + s;
        q[r] = reinterpret_cast<const float4*>(a.qrot + orow * 128)[lane];
      }
    }
  }
  float m[kRB], l[kRB];
  float4 acc[kRB];
#pragma unroll
  for (int r = 0; r < kRB; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
    acc[r] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const T* kb = static_cast<const T*>(a.k) + (a.B > 1 ? int64_t(b) * a.k_sb : 0) + int64_t(h) * a.k_sh;
  const T* vb = static_cast<const T*>(a.v) + (a.B > 1 ? int64_t(b) * a.v_sb : 0) + int64_t(h) * a.v_sh;
  // the warp's contiguous share of the split, kU = 32 / kRB keys at a time: one
  // load brings the kU positions (lane u holds key jb + u), then all kU key and
  // value rows are requested before the first is used. The kU x kRB dot products
  // are reduced across the warp together (a transposed butterfly: 31 shuffles for
  // 32 sums; lane l ends with the score of key l / kRB for row l % kRB), so each
  // lane runs the softmax bookkeeping of one (key, row) pair, and the group's
  // running maximum is folded in once per row.
  constexpr int kU = 32 / kRB;
  float lpart = 0.f;  // this lane's share of l[lane % kRB]
  const int my_u = lane / kRB, my_r = lane % kRB;
  const int64_t wper = (j1 - j0 + kSaWarps - 1) / kSaWarps;
  const int64_t w0 = j0 + int64_t(warp) * wper;
  const int64_t w1 = w0 + wper < j1 ? w0 + wper : j1;
  for (int64_t jb = w0; jb < w1; jb += kU) {
    const int64_t mine = jb + lane;
    const int64_t pos = lane < kU && mine < w1 ? a.key_pos[mine] : -1;
    uint2 kraw[kU], vraw[kU];  // packed 16-bit rows
    int pu[kU];                // positions (< S < 2^31); -1: no key
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t pp = __shfl_sync(0xffffffffu, pos, u);
      const bool ok = jb + u < w1 && pp >= 0 && pp < a.S;
      if (jb + u < w1 && !ok && lane == 0) set_status(a.status, kStatusBounds);  // skipped
      pu[u] = ok ? int(pp) : -1;
      kraw[u] = ok ? *reinterpret_cast<const uint2*>(kb + pp * 128 + 4 * lane) : make_uint2(0u, 0u);
      vraw[u] = ok ? *reinterpret_cast<const uint2*>(vb + pp * 128 + 4 * lane) : make_uint2(0u, 0u);
    }
    // partial dot products: d[u * kRB + r] = this lane's 4 dimensions of q_r . k_u
    float d[32];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      float4 kf;
      Unpack<T>::run(kraw[u].x, kf.x, kf.y);
      Unpack<T>::run(kraw[u].y, kf.z, kf.w);
      if (kRope) kf = rope4_table(kf, a.table + (jb + u < w1 ? (jb + u) : w0) * 64, lane);
#pragma unroll
      for (int r = 0; r < kRB; ++r) d[u * kRB + r] = dot4(q[r], kf);
    }
    // transposed butterfly: lane l ends with the full sum of d[l]
#pragma unroll
    for (int o = 16, n = 32; o >= 1; o >>= 1, n >>= 1) {
      const bool up = lane & o;
#pragma unroll
      for (int i = 0; i < n / 2; ++i) {
        const float send = up ? d[i] : d[i + n / 2];
        const float keep = up ? d[i + n / 2] : d[i];
        d[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
      }
    }
    const int pk = pu_at(pu, my_u);  // position of this lane's key
    const bool live = pk >= 0 && my_r < nrows && int64_t(pk) <= qabs_at(qabs, my_r);
    const float sc = live ? d[0] : -INFINITY;
    // the group's maximum per row (lanes with the same row differ in bits >= log2(kRB))
    float gm = sc;
#pragma unroll
    for (int o = kRB; o < 32; o <<= 1) gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, o));
    float corr_r[kRB];
#pragma unroll
    for (int r = 0; r < kRB; ++r) {
      const float mn = fmaxf(m[r], __shfl_sync(0xffffffffu, gm, r));
      corr_r[r] = mn == -INFINITY ? 1.f : __expf(m[r] - mn);
      m[r] = mn;
    }
    const float e = live ? __expf(sc - pick<kRB, float>(m, my_r)) : 0.f;
    lpart = fmaf(lpart, pick<kRB, float>(corr_r, my_r), e);
#pragma unroll
    for (int r = 0; r < kRB; ++r) {
      acc[r].x *= corr_r[r];
      acc[r].y *= corr_r[r];
      acc[r].z *= corr_r[r];
      acc[r].w *= corr_r[r];
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      float4 vf;
      Unpack<T>::run(vraw[u].x, vf.x, vf.y);
      Unpack<T>::run(vraw[u].y, vf.z, vf.w);
#pragma unroll
      for (int r = 0; r < kRB; ++r) {
        const float eu = __shfl_sync(0xffffffffu, e, u * kRB + r);
        acc[r].x = fmaf(eu, vf.x, acc[r].x);
        acc[r].y = fmaf(eu, vf.y, acc[r].y);
        acc[r].z = fmaf(eu, vf.z, acc[r].z);
        acc[r].w = fmaf(eu, vf.w, acc[r].w);
      }
    }
  }
  // l[r]: the lanes of row r hold its parts
#pragma unroll
  for (int o = kRB; o < 32; o <<= 1) lpart += __shfl_xor_sync(0xffffffffu, lpart, o);
#pragma unroll
  for (int r = 0; r < kRB; ++r) l[r] = __shfl_sync(0xffffffffu, lpart, r);
#pragma unroll
  for (int r = 0; r < kRB; ++r) {
    if (lane == 0) {
      s_m[warp][r] = m[r];
      s_l[warp][r] = l[r];
    }
    s_acc[warp][r][lane] = acc[r];
  }
  __syncthreads();
  // merge the warps: warp w merges rows w, w + 8, ... (one row per warp here)
  for (int r = warp; r < nrows; r += kSaWarps) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kSaWarps; ++w) M = fmaxf(M, s_m[w][r]);
    float L = 0.f;
    float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kSaWarps; ++w) {
        const float f = __expf(s_m[w][r] - M);
        L = fmaf(s_l[w][r], f, L);
        const float4 x = s_acc[w][r][lane];
        A.x = fmaf(x.x, f, A.x);
        A.y = fmaf(x.y, f, A.y);
        A.z = fmaf(x.z, f, A.z);
        A.w = fmaf(x.w, f, A.w);
      }
    }
    const int64_t rr = r0 + r, g = rr / a.Sq, s = rr - g * a.Sq;
    const int64_t orow = (int64_t(b) * a.Hq + int64_t(h) * a.G + g) * a.Sq + s;
    const int64_t slot = orow * nsplit + split;
    if (lane == 0) {
      a.part_m[slot] = M;
      a.part_l[slot] = L;
    }
    reinterpret_cast<float4*>(a.part_acc + slot * 128)[lane] = A;
  }
}

// Merge of the splits: kWpr warps per row (8 when the row has many splits, 1
// otherwise). Every warp of the row takes the row maximum over all splits (one
// load per lane), then folds its splits sp = sub, sub + kWpr, ... four at a time
// with all their loads in flight; the row's warps are summed in shared memory.
template <typename T, int kWpr>
__global__ void __launch_bounds__(256) sparse_attn_combine_kernel(const SparseAttnArgs a, int nsplit) {
  constexpr int kRpc = 8 / kWpr;  // rows per CTA
  __shared__ float s_l[8];
  __shared__ float4 s_acc[8][32];
  // programmatic dependent launch: the partials are complete and visible after this
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = warp % kWpr;
  const int64_t row = int64_t(blockIdx.x) * kRpc + warp / kWpr;
  const int64_t rows = int64_t(a.B) * a.Hq * a.Sq;
  const bool ok = row < rows;
  const int64_t base = row * nsplit;
  float M = -INFINITY;
  if (ok) {
#pragma unroll
    for (int t = 0; t < kSparseMaxSplits / 32; ++t)
      if (lane + 32 * t < nsplit) M = fmaxf(M, a.part_m[base + lane + 32 * t]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  float L = 0.f;
  float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
  if (ok && M != -INFINITY) {
    for (int sp0 = sub; sp0 < nsplit; sp0 += 4 * kWpr) {
      float mm[4], ll[4];
      float4 xx[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int sp = sp0 + u * kWpr;
        mm[u] = -INFINITY;
        ll[u] = 0.f;
        xx[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (sp < nsplit) {
          mm[u] = a.part_m[base + sp];
          ll[u] = a.part_l[base + sp];
          xx[u] = reinterpret_cast<const float4*>(a.part_acc + (base + sp) * 128)[lane];
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float f = __expf(mm[u] - M);
        L = fmaf(ll[u], f, L);
        A.x = fmaf(xx[u].x, f, A.x);
        A.y = fmaf(xx[u].y, f, A.y);
        A.z = fmaf(xx[u].z, f, A.z);
        A.w = fmaf(xx[u].w, f, A.w);
      }
    }
  }
  if (kWpr > 1) {
    if (lane == 0) s_l[warp] = L;
    s_acc[warp][lane] = A;
    __syncthreads();
    if (sub != 0) return;
    L = 0.f;
    A = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < kWpr; ++w) {
      L += s_l[warp + w];
      const float4 x = s_acc[warp + w][lane];
      A.x += x.x;
      A.y += x.y;
      A.z += x.z;
      A.w += x.w;
    }
  }
  if (!ok) return;
  // a row that sees no key gets zeros (the reference's nan_to_num of 0/0)
  const float inv = L > 0.f ? 1.f / L : 0.f;
  A.x *= inv;
  A.y *= inv;
  A.z *= inv;
  A.w *= inv;
  store4<T>(static_cast<T*>(a.out) + row * 128 + 4 * lane, A);
}

// (cos, sin) of every view position's 64 RoPE angles, fp32(pe) * inv_freq[i]
// evaluated with the accurate reduction of rope_sincos.cuh: [nsel][64] float2;
// the threads past the table rotate the query rows at their positions and scale
// them: qrot[row][i], qrot[row][i + 64] (fp32), row = (b * Hq + hq) * Sq + s.
template <typename T>
__global__ void rope_table_kernel(const SparseAttnArgs a, float2* table, float* qrot) {
  asm volatile("griddepcontrol.launch_dependents;");
  const int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t ntab = a.nsel * 64;
  const int64_t rows = int64_t(a.B) * a.Hq * a.Sq;
  if (e < ntab) {
    const int64_t j = e >> 6;
    const int i = int(e & 63);
    const float pe = a.pe_original ? float(a.key_pos[j]) : float(j);
    float sn, cs;
    rope_sincos(__fmul_rn(pe, a.inv_freq[i]), sn, cs);
    table[e] = make_float2(cs, sn);
    return;
  }
  const int64_t f = e - ntab;
  if (f >= rows * 64) return;
  const int64_t row = f >> 6;
  const int i = int(f & 63);
  const int64_t s = row % a.Sq, bh = row / a.Sq, hq = bh % a.Hq, b = bh / a.Hq;
  const T* qr = static_cast<const T*>(a.q) + b * a.q_sb + hq * a.q_sh + s * a.q_ss;
  const float x0 = to_f32(qr[i]), x1 = to_f32(qr[i + 64]);
  const float pe = a.pe_original ? float(a.q_pos[s]) : float(a.nsel - a.Sq + s);
  float sn, cs;
  rope_sincos(__fmul_rn(pe, a.inv_freq[i]), sn, cs);
  qrot[row * 128 + i] = (x0 * cs - x1 * sn) * a.scale;
  qrot[row * 128 + i + 64] = (x1 * cs + x0 * sn) * a.scale;
}

int sa_rows(const SparseAttnArgs& a) { return int64_t(a.G) * a.Sq <= 4 ? 4 : 8; }

// splits of the view the workspace holds room for: up to kSparseMaxSplits, and
// at most 8192 (row, split) partials beyond one per row
int64_t split_cap(int64_t rows) {
  const int64_t c = 8192 / (rows > 0 ? rows : 1);
  return c < 1 ? 1 : (c < kSparseMaxSplits ? c : kSparseMaxSplits);
}

int sa_splits(const SparseAttnArgs& a, int num_sms) {
  const int64_t R = int64_t(a.G) * a.Sq;
  const int rb = sa_rows(a);
  const int64_t ctas = int64_t(a.B) * a.Hkv * ((R + rb - 1) / rb);
  int64_t s = (int64_t(num_sms) * 4 + ctas - 1) / ctas;  // about four CTAs per SM
  const int64_t maxs = (a.nsel + 255) / 256;            // at least 256 keys per split
  s = s < maxs ? s : maxs;
  const int64_t cap = split_cap(int64_t(a.B) * a.Hq * a.Sq);
  s = s < cap ? s : cap;
  return int(s < 1 ? 1 : s);
}

// The partial kernel follows the angle table with a dependent launch when there
// is one (it reads only the caller's inputs before its wait); without RoPE it
// follows the caller's own work and launches normally.
template <typename T, bool kRope>
cudaError_t launch_partial(const SparseAttnArgs& a, int nsplit, cudaStream_t stream) {
  const int64_t R = int64_t(a.G) * a.Sq;
  const int rb = sa_rows(a);
  const dim3 grid(unsigned(int64_t(a.B) * a.Hkv * ((R + rb - 1) / rb)), unsigned(nsplit));
  if (rb == 4)
    return launch_maybe_dependent(sparse_attn_partial_kernel<T, kRope, 4>, grid, dim3(kSaWarps * 32), 0, kRope,
                            stream, a);
  return launch_maybe_dependent(sparse_attn_partial_kernel<T, kRope, 8>, grid, dim3(kSaWarps * 32), 0, kRope,
                          stream, a);
}

template <typename T>
cudaError_t launch_combine(const SparseAttnArgs& a, int nsplit, cudaStream_t stream) {
  const int64_t rows = int64_t(a.B) * a.Hq * a.Sq;
  if (nsplit > 4)
    return launch_maybe_dependent(sparse_attn_combine_kernel<T, 8>, dim3(unsigned(rows)), dim3(256), 0, true,
                            stream, a, nsplit);
  return launch_maybe_dependent(sparse_attn_combine_kernel<T, 1>, dim3(unsigned((rows + 7) / 8)), dim3(256), 0,
                                true, stream, a, nsplit);
}

template <typename T>
cudaError_t launch_attn(const SparseAttnArgs& a, int nsplit, cudaStream_t stream) {
  cudaError_t e = a.inv_freq != nullptr ? launch_partial<T, true>(a, nsplit, stream)
                                        : launch_partial<T, false>(a, nsplit, stream);
  if (e != cudaSuccess) return e;
  return launch_combine<T>(a, nsplit, stream);
}

}  // namespace

size_t sparse_attn_workspace_bytes(int64_t B, int64_t Hq, int64_t Sq, int64_t nsel) {
  const size_t rows = size_t(B) * size_t(Hq) * size_t(Sq);
  return (rows * size_t(split_cap(int64_t(rows))) * (2 + 128) * sizeof(float) + 255) / 256 * 256 +
         (size_t(nsel) * 64 * sizeof(float2) + 255) / 256 * 256 + rows * 128 * sizeof(float);
}

cudaError_t launch_sparse_attn(SparseAttnArgs a, int dtype, void* ws, int num_sms,
                               cudaStream_t stream) {
  const int nsplit = sa_splits(a, num_sms);
  const size_t rows = size_t(a.B) * size_t(a.Hq) * size_t(a.Sq);
  const size_t cap = size_t(split_cap(int64_t(rows)));
  float* w = static_cast<float*>(ws);
  a.part_m = w;
  a.part_l = w + rows * cap;
  a.part_acc = w + 2 * rows * cap;
  const size_t tab_off = (rows * cap * (2 + 128) * sizeof(float) + 255) / 256 * 256;
  float2* table = reinterpret_cast<float2*>(static_cast<uint8_t*>(ws) + tab_off);
  float* qrot = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + tab_off +
                                         (size_t(a.nsel) * 64 * sizeof(float2) + 255) / 256 * 256);
  if (a.inv_freq != nullptr) {
    const int64_t n = (a.nsel + int64_t(rows)) * 64;
    if (dtype == kBF16)
      rope_table_kernel<__nv_bfloat16><<<unsigned((n + 255) / 256), 256, 0, stream>>>(a, table, qrot);
    else
      rope_table_kernel<__half><<<unsigned((n + 255) / 256), 256, 0, stream>>>(a, table, qrot);
    a.table = table;
    a.qrot = qrot;
  }
  const cudaError_t e = dtype == kBF16 ? launch_attn<__nv_bfloat16>(a, nsplit, stream)
                                        : launch_attn<__half>(a, nsplit, stream);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace prism
