// Host side of the TMA helpers: tensor-map encoding through the driver entry point
// (no link-time dependency on libcuda).
#include <mutex>

#include "tma.cuh"

namespace pyre {
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

}  // namespace

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t rows,
                 uint64_t cols, uint64_t row_stride_bytes, uint32_t box_rows, uint32_t box_cols,
                 CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return set_error(PYRE_ECUDA, "cuTensorMapEncodeTiled entry point unavailable");
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return set_error(PYRE_EINVAL, "TMA base address must be 16-byte aligned");
  if (row_stride_bytes % 16 != 0) return set_error(PYRE_EINVAL, "TMA row stride must be a multiple of 16 bytes");
  if ((static_cast<uint64_t>(box_cols) * elem_bytes) % 16 != 0)
    return set_error(PYRE_EINVAL, "TMA box inner extent must be a multiple of 16 bytes");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(PYRE_EINVAL, "cuTensorMapEncodeTiled failed (code " + std::to_string(r) + ")");
  return PYRE_OK;
}

int make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t d0,
                 uint64_t d1, uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0,
                 uint32_t box1, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return set_error(PYRE_ECUDA, "cuTensorMapEncodeTiled entry point unavailable");
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return set_error(PYRE_EINVAL, "TMA base address must be 16-byte aligned");
  if (stride1_bytes % 16 != 0 || stride2_bytes % 16 != 0)
    return set_error(PYRE_EINVAL, "TMA strides must be multiples of 16 bytes");
  if ((static_cast<uint64_t>(box0) * elem_bytes) % 16 != 0)
    return set_error(PYRE_EINVAL, "TMA box inner extent must be a multiple of 16 bytes");
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {box0, box1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dtype, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(PYRE_EINVAL, "cuTensorMapEncodeTiled failed (code " + std::to_string(r) + ")");
  return PYRE_OK;
}

}  // namespace pyre
