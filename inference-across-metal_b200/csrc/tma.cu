// Host side of the TMA helpers: tensor-map encoding through the driver entry
// point (no link-time dependency on libcuda).
#include <mutex>

#include "tma.cuh"

namespace iam {
namespace {

typedef CUresult (*EncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  });
  return fn;
}

}  // namespace

int tma_encode_2d(CUtensorMap* map, const void* base, int esize, uint64_t rows, uint64_t cols, uint32_t box_rows,
                  uint32_t box_cols, bool swizzle128, uint64_t pitch) {
  EncodeTiled fn = encoder();
  if (!fn) return fail(IAM_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  IAM_CHECK(aligned16(base), "tma: base must be 16-byte aligned");
  if (pitch == 0) pitch = cols;
  IAM_CHECK(pitch >= cols && (pitch * esize) % 16 == 0, "tma: row pitch must be a multiple of 16 bytes");
  IAM_CHECK((box_cols * esize) % 16 == 0 && box_cols <= 256 && box_rows <= 256, "tma: bad box");
  IAM_CHECK(!swizzle128 || box_cols * esize <= 128, "tma: swizzled box wider than 128 bytes");
  const CUtensorMapDataType dt = esize == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                            : (esize == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT32);
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {pitch * esize};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(IAM_EINVAL, "cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  return IAM_OK;
}

}  // namespace iam
