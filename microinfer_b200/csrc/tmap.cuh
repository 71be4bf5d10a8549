// Host-side TMA tensor-map encoding shared by the kernels.
//
// The pool and the query/output tensors are all addressed as 3-D maps
// x = head dimension (contiguous), y = heads, z = rows (tokens or pool
// slots), so a box {x, 1, n} fetches n rows of one head in one request.
// cuTensorMapEncodeTiled comes from the driver through cudaGetDriverEntryPoint
// (no link-time dependency on libcuda).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>

namespace mi {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 3-D map over [rows][heads][d] with a {box_x, box_y, box_z} box.  Returns
// false when the driver entry point is missing or the encoding is rejected.
inline bool encode_rows_map(CUtensorMap *map, CUtensorMapDataType dt, const void *base, uint64_t d,
                            uint64_t heads, uint64_t rows, uint64_t head_stride_bytes,
                            uint64_t row_stride_bytes, uint32_t box_x, uint32_t box_y,
                            uint32_t box_z, CUtensorMapSwizzle swizzle) {
  auto fn = tensor_map_encoder();
  if (fn == nullptr) return false;
  cuuint64_t dims[3] = {d, heads, rows};
  cuuint64_t strides[2] = {head_stride_bytes, row_stride_bytes};
  cuuint32_t box[3] = {box_x, box_y, box_z};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, dt, 3, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace mi
