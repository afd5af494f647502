// Fifth-generation tensor-core primitives for sm_100a (inline PTX): tensor
// memory (TMEM) allocation, tcgen05.mma with shared-memory operand descriptors,
// commit to an mbarrier, and TMEM -> register loads.
//
// Operand layout used throughout: K-major tiles of 16-bit elements in the
// 128-byte swizzle mode — rows of 64 elements (128 B), grouped in 8-row atoms of
// 1024 B whose 16-byte chunks are XOR-permuted by the row's index within the
// atom (chunk c of row r sits at chunk c ^ (r & 7)). This is what a TMA tile
// copy with CU_TENSOR_MAP_SWIZZLE_128B and a 64-element inner box writes, and
// what the descriptor below describes (stride between 8-row groups: 1024 B).
#pragma once

#include "common.cuh"

namespace prism {

// ---- tensor memory -----------------------------------------------------------------
// One full warp executes alloc / relinquish / dealloc. The allocated column base
// (lane 0, column base) is written to *dst in shared memory.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// Ordering of tcgen05 operations across thread synchronisation (mbarriers,
// bar.sync): "before" on the releasing side, "after" on the acquiring side.
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Generic-proxy writes to shared memory made visible to the async proxy (the
// tensor cores read operands through it).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- descriptors ---------------------------------------------------------------------
// Shared-memory matrix descriptor of a K-major, 128-byte-swizzled operand tile
// starting at shared address `saddr` (the tile's 8-row atoms 1024 B apart).
// Bits: [0,14) start >> 4; [16,30) leading byte offset >> 4 (unused by swizzled
// K-major layouts, set to 1); [32,46) stride byte offset >> 4 = 1024 >> 4;
// [46,48) descriptor version 1; [49,52) base offset 0 (atoms 1024-byte aligned);
// [61,64) layout 2 = 128-byte swizzle. Stepping K by 16 elements (32 B) inside an
// atom adds 2 to the start field.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
  uint64_t d = uint64_t((saddr >> 4) & 0x3FFFu);
  d |= uint64_t(1) << 16;
  d |= uint64_t(1024 >> 4) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(2) << 61;
  return d;
}

// Instruction descriptor of tcgen05.mma kind::f16: fp32 accumulator, A and B of
// the same 16-bit type (bf16 or fp16), both K-major, M x N tile.
// Bits: [4,6) D format 1 = f32; [7,10) A format; [10,13) B format (0 f16, 1 bf16);
// 15 / 16 A / B major (0 = K); [17,23) N >> 3; [24,29) M >> 4.
__host__ __device__ constexpr uint32_t idesc_kind_f16(bool bf16, int M, int N) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
         (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

// ---- MMA, commit, TMEM loads ------------------------------------------------------------
// D[tmem] (+)= A[smem] * B[smem]^T for one K = 16 step; issued by one thread.
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once) on `bar` when every tcgen05.mma this thread issued so far has
// completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 consecutive 32-bit columns of this warp's 32 TMEM lanes (lane i of the
// warp reads TMEM lane (taddr >> 16) + i). Complete with tmem_ld_wait().
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

}  // namespace prism
