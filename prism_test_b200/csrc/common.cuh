// Shared device helpers for the ReAttention recall scorer (sm_100a).
//
// Everything here is plain CUDA C++ plus hand-written inline PTX for the
// Blackwell/Hopper asynchronous-copy machinery (mbarrier + cp.async.bulk).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace prism {

constexpr int kHeadDim = 128;          // head_dim handled by every kernel
constexpr int kRowBytes = kHeadDim * 2;  // one bf16/fp16 key row

// Device status word values (written by kernels, read by the host on demand).
enum : int {
  kStatusOk = 0,
  kStatusTimeout = 1,    // a bounded wait on an mbarrier / peer flag expired
  kStatusBounds = 2,     // a kernel-side bounds check rejected an access
  kStatusCapacity = 3,   // a candidate buffer would have overflowed
};

// Bounded waits give up after this many nanoseconds of %globaltimer.
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;  // 2 s

__device__ __forceinline__ void set_status(int* status, int code) {
  if (status != nullptr) atomicCAS(status, kStatusOk, code);
}

// ---------------------------------------------------------------------------
// Order-preserving 32-bit key of an fp32 score: larger float -> larger key.
// NaN maps to the largest key (torch.topk treats NaN as the largest value).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t float_to_okey(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0xffffffffu;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float okey_to_float(uint32_t k) {
  if (k == 0xffffffffu) return __uint_as_float(0x7fc00000u);
  uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

// ---------------------------------------------------------------------------
// Shared-memory / mbarrier / bulk-copy primitives (inline PTX).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for the phase with the given parity to complete. Returns false (and the
// caller must set an error status and bail out) after kWaitTimeoutNs.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > kWaitTimeoutNs) return false;
  }
}

// The same wait for roles with many waiting threads: try_wait with a suspend-time
// hint, so that a waiting thread sleeps until the phase completes (or the hint
// runs out) instead of polling the barrier in shared memory.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(100000u)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_sleep_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait_sleep(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait_sleep(bar, parity))
    if (globaltimer_ns() - t0 > kWaitTimeoutNs) return false;
  return true;
}

// L2 policy: stream-once data (the key cache) is marked evict-first so that
// the score buffer written alongside it stays resident in L2.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// 1-D bulk copy global -> shared, completing on an mbarrier (TMA engine).
// Both addresses must be 16-byte aligned and bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Tiled 4-D tensor copy global -> shared (TMA), completing on an mbarrier. The
// tensor map lives in kernel parameter space (__grid_constant__); the copy lands
// only in this CTA's shared memory.
__device__ __forceinline__ void tma_load_4d(void* smem_dst, const void* tmap, int c0, int c1, int c2,
                                            int c3, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(smem_dst)),
      "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint4 lds128(const void* p) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(smem_u32(p)));
  return v;
}

// 128-bit shared loads from a 32-bit shared-window address
__device__ __forceinline__ uint4 lds128_u32(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}
__device__ __forceinline__ uint2 lds64_u32(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}
__device__ __forceinline__ float4 lds128f_u32(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr));
  return v;
}

// ---------------------------------------------------------------------------
// Packed 16-bit -> fp32 unpacking. A 32-bit word holds elements (lo, hi).
// ---------------------------------------------------------------------------
template <typename T>
struct Unpack;
template <>
struct Unpack<__nv_bfloat16> {
  __device__ __forceinline__ static void run(uint32_t w, float& lo, float& hi) {
    lo = __uint_as_float(w << 16);
    hi = __uint_as_float(w & 0xffff0000u);
  }
};
template <>
struct Unpack<__half> {
  __device__ __forceinline__ static void run(uint32_t w, float& lo, float& hi) {
    __half2 h = *reinterpret_cast<__half2*>(&w);
    float2 f = __half22float2(h);
    lo = f.x;
    hi = f.y;
  }
};

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) {
  return __half2float(v);
}

// Programmatic dependent launch: wait until the kernel before this one in the
// stream has completed and its writes are visible; a no-op for a normal launch.
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Launches kern<<<grid, block, smem, stream>>>(args...), as a programmatic
// dependent launch when pdl: the kernel may be scheduled while the previous
// kernel in the stream drains, and must read that kernel's output only after
// its griddepcontrol.wait.
template <typename... P, typename... A>
cudaError_t launch_maybe_dependent(void (*kern)(P...), dim3 grid, dim3 block, size_t smem, bool pdl,
                                   cudaStream_t stream, A... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

}  // namespace prism
