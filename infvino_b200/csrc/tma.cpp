#include "tma.h"

#include <cuda_runtime.h>
#include <mutex>

namespace ivb {

namespace {
using EncodeFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                              const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn get_encode(std::string *err) {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  static std::string init_err;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    const cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p)
      init_err = "cuTensorMapEncodeTiled unavailable";
    else
      fn = reinterpret_cast<EncodeFn>(p);
  });
  if (!fn && err) *err = init_err;
  return fn;
}
}  // namespace

CUtensorMapSwizzle swizzle_for_row_bytes(int row_bytes) {
  if (row_bytes == 128) return CU_TENSOR_MAP_SWIZZLE_128B;
  if (row_bytes == 64) return CU_TENSOR_MAP_SWIZZLE_64B;
  return CU_TENSOR_MAP_SWIZZLE_32B;
}

bool encode_tiled_f16(CUtensorMap *map, int rank, const void *base, const uint64_t *dims,
                      const uint64_t *byte_strides, const uint32_t *box, const uint32_t *elem_strides,
                      CUtensorMapSwizzle swizzle, std::string *err) {
  EncodeFn fn = get_encode(err);
  if (!fn) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) {
    if (err) *err = "tensor map base not 16-byte aligned";
    return false;
  }
  for (int i = 0; i + 1 < rank; ++i)
    if (byte_strides[i] % 16 != 0) {
      if (err) *err = "tensor map stride not a multiple of 16 bytes";
      return false;
    }
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, (cuuint32_t)rank, const_cast<void *>(base),
                        reinterpret_cast<const cuuint64_t *>(dims), reinterpret_cast<const cuuint64_t *>(byte_strides),
                        reinterpret_cast<const cuuint32_t *>(box), reinterpret_cast<const cuuint32_t *>(elem_strides),
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    if (err) *err = "cuTensorMapEncodeTiled failed with code " + std::to_string((int)r);
    return false;
  }
  return true;
}

}  // namespace ivb
