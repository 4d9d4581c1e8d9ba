// Host-side helpers: TMA tensor-map encoding through the driver entry point
// (looked up lazily through the runtime, so importing an extension does not
// need libcuda on machines without a GPU), device SM count cache, and
// argument checks shared by the op launchers.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <stdexcept>
#include <string>

namespace b200 {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn get_encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr) {
      throw std::runtime_error("b200: cannot resolve cuTensorMapEncodeTiled from the CUDA driver");
    }
    fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D tiled map over a row-major matrix [rows, cols] (cols contiguous) with a
// box of [box_rows, box_cols] elements and 128-byte swizzle. box_cols *
// elem_bytes must equal 128 for the swizzle span used by the UMMA layouts.
inline CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t rows,
                                uint64_t cols, uint64_t row_stride_elems, uint32_t box_rows, uint32_t box_cols,
                                CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) throw std::runtime_error("b200: TMA base not 16B aligned");
  if ((row_stride_elems * elem_bytes) % 16 != 0) throw std::runtime_error("b200: TMA row stride not 16B multiple");
  CUtensorMap m;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_elems * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode_tiled()(&m, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("b200: cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return m;
}

// 3-D tiled map over [d2][d1][d0] (d0 contiguous; strides in elements for d1
// and d2) with box [b2][b1][b0] and 128-byte swizzle.
inline CUtensorMap make_tmap_3d(const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t d0, uint64_t d1,
                                uint64_t d2, uint64_t stride1_elems, uint64_t stride2_elems, uint32_t b0, uint32_t b1,
                                uint32_t b2, CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) throw std::runtime_error("b200: TMA base not 16B aligned");
  if ((stride1_elems * elem_bytes) % 16 != 0 || (stride2_elems * elem_bytes) % 16 != 0)
    throw std::runtime_error("b200: TMA strides not 16B multiples");
  CUtensorMap m;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_elems * (uint64_t)elem_bytes, stride2_elems * (uint64_t)elem_bytes};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = get_encode_tiled()(&m, dtype, 3, const_cast<void*>(base), dims, strides, box, estr,
                                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("b200: cuTensorMapEncodeTiled (3d) failed: " + std::to_string((int)r));
  return m;
}

inline int num_sms(int device) {
  static int cache[64] = {0};
  if (device < 0 || device >= 64) device = 0;
  if (cache[device] == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device);
    cache[device] = v > 0 ? v : 148;
  }
  return cache[device];
}

}  // namespace b200
