// Host-side construction of TMA tensor maps (cuTensorMapEncodeTiled, obtained
// from the driver through the runtime so the library needs no -lcuda).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>

namespace prism {

// 4-D map over a key cache [B, Hkv, Sk, 128] of 2-byte elements with element
// strides (k_sb, k_sh, 128, 1); box {128, box_rows, box_heads, 1} (box_heads <= 0
// means all Hkv heads). Rows beyond Sk are zero-filled. A batch stride of 0
// (broadcast keys) maps every batch to b = 0. Returns cudaErrorInvalidValue when
// the driver rejects the description.
cudaError_t make_key_tensor_map(CUtensorMap* map, const void* k, int dtype, int64_t B, int64_t Hkv,
                                int64_t Sk, int64_t k_sb, int64_t k_sh, int box_rows,
                                int box_heads = 0);

// The same key cache as a K-major tensor-core operand: box {64, 128, 1, 1} (64
// dimensions x 128 positions of one KV head = one 16 KB atom per copy), written
// to shared memory in the 128-byte swizzle mode. With key_stride s > 1 the map
// covers only every s-th key (positions 0, s, 2s, ...): a strided sample.
cudaError_t make_key_tensor_map_sw128(CUtensorMap* map, const void* k, int dtype, int64_t B,
                                      int64_t Hkv, int64_t Sk, int64_t k_sb, int64_t k_sh,
                                      int key_stride = 1);

}  // namespace prism
