// Host-side access to cuTensorMapEncodeTiled through the runtime's driver
// entry-point query (no link dependency on libcuda).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

namespace tssm {

inline PFN_cuTensorMapEncodeTiled_v12000 tmap_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 3-D f32 map over [d2][d1][d0] (d0 contiguous), box {b0, b1, 1}, no swizzle;
// out-of-range rows read as zero and are not written.
inline bool tmap3d_f32(CUtensorMap* m, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint32_t b0,
                       uint32_t b1) {
  auto fn = tmap_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {d0 * 4, d0 * d1 * 4};
  cuuint32_t box[3] = {b0, b1, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D f32 map over [d1][d0] (d0 contiguous, row pitch d0*4 bytes) with a
// {32, b1} box in the 128B swizzle (one 128-byte row of the box per d1 index);
// out-of-range elements read as zero and are not written.
inline bool tmap2d_f32_sw128(CUtensorMap* m, const void* base, uint64_t d0, uint64_t d1, uint32_t b1) {
  auto fn = tmap_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {d0, d1};
  cuuint64_t strides[1] = {d0 * 4};
  cuuint32_t box[2] = {32, b1};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tssm
