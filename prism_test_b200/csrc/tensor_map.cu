#include <mutex>

#include "kernels.h"
#include "tensor_map.h"

namespace prism {
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

}  // namespace

cudaError_t make_key_tensor_map(CUtensorMap* map, const void* k, int dtype, int64_t B, int64_t Hkv,
                                int64_t Sk, int64_t k_sb, int64_t k_sh, int box_rows,
                                int box_heads) {
  PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
  if (fn == nullptr) return cudaErrorNotSupported;
  const bool batched = B > 1 && k_sb != 0;
  cuuint64_t dims[4] = {128, cuuint64_t(Sk), cuuint64_t(Hkv), cuuint64_t(batched ? B : 1)};
  cuuint64_t strides[3] = {256, cuuint64_t(k_sh) * 2,
                           cuuint64_t(batched ? k_sb : k_sh * Hkv) * 2};
  cuuint32_t box[4] = {128, cuuint32_t(box_rows), cuuint32_t(box_heads > 0 ? box_heads : Hkv), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt =
      dtype == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(map, dt, 4, const_cast<void*>(k), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t make_key_tensor_map_sw128(CUtensorMap* map, const void* k, int dtype, int64_t B,
                                      int64_t Hkv, int64_t Sk, int64_t k_sb, int64_t k_sh,
                                      int key_stride) {
  PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
  if (fn == nullptr) return cudaErrorNotSupported;
  const bool batched = B > 1 && k_sb != 0;
  const int64_t nkeys = (Sk + key_stride - 1) / key_stride;
  cuuint64_t dims[4] = {128, cuuint64_t(nkeys), cuuint64_t(Hkv), cuuint64_t(batched ? B : 1)};
  cuuint64_t strides[3] = {cuuint64_t(256) * cuuint64_t(key_stride), cuuint64_t(k_sh) * 2,
                           cuuint64_t(batched ? k_sb : k_sh * Hkv) * 2};
  cuuint32_t box[4] = {64, 128, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt =
      dtype == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(map, dt, 4, const_cast<void*>(k), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace prism
