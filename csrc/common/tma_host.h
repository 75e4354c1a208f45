// Host-side helpers: tensor-map encoding through the driver entry point (no -lcuda link
// dependency) and cached device properties.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <algorithm>
#include <mutex>
#include <stdexcept>
#include <string>

namespace gollek {

// Status buffer of the device bounds checks (uint32 [2]: status bits, first bad index), or nullptr
// when checking is off. One slot per process (an inline function's static), set from Python.
inline uint32_t*& bounds_status_slot() {
  static uint32_t* p = nullptr;
  return p;
}
inline uint32_t* bounds_status() { return bounds_status_slot(); }

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn get_encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr)
      throw std::runtime_error("cannot resolve cuTensorMapEncodeTiled from the CUDA driver");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D row-major tensor [rows, cols] of `elem_bytes` elements with row pitch `ld` elements.
// Box = [box_cols, box_rows]; box_cols * elem_bytes must be 16-byte multiple (128 with SW128).
inline CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t rows,
                                uint64_t cols, uint64_t ld, uint32_t box_rows, uint32_t box_cols,
                                CUtensorMapSwizzle swizzle) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) throw std::runtime_error("TMA base address must be 16-byte aligned");
  if ((ld * elem_bytes) % 16 != 0) throw std::runtime_error("TMA row pitch must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode_tiled()(&m, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed with code " + std::to_string((int)r));
  return m;
}

inline int num_sms() {
  static int n = 0;
  static std::once_flag once;
  std::call_once(once, [] {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  });
  return n;
}

// SMs kept free of the persistent GEMM grids (0 = none). While a collective of one half of a
// split batch runs on another stream, the GEMMs of the other half leave it these SMs.
inline int& gemm_sm_reserve() {
  static int r = 0;
  return r;
}
inline int gemm_grid_sms() { return std::max(1, num_sms() - gemm_sm_reserve()); }

}  // namespace gollek
