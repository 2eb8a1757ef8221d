// Host-side helpers for the TMA kernels: tensor-map encoding through the
// driver entry point (no link-time libcuda dependency) and layout checks.
#pragma once

#include <cuda.h>

#include <mutex>
#include <string>

#include "common.cuh"

namespace poly {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 4-D tiled map over a [batch, heads, rows, d] tensor with (b, h, row) element
// strides; box = 64 features x box_rows rows, 128-byte swizzle.
inline int make_map(CUtensorMap* m, const void* base, int dtype, int d, int rows, int heads, int batch,
             const int64_t* st, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is unavailable");
    return POLY_ECUDA;
  }
  const cuuint64_t dims[4] = {(cuuint64_t)d, (cuuint64_t)rows, (cuuint64_t)heads, (cuuint64_t)batch};
  const cuuint64_t strides[3] = {(cuuint64_t)st[2] * 2, (cuuint64_t)st[1] * 2, (cuuint64_t)st[0] * 2};
  const cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  const cuuint32_t es[4] = {1, 1, 1, 1};
  const CUresult r = fn(m, dtype == POLY_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                        const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    return POLY_ECUDA;
  }
  return POLY_OK;
}

// 3-D fp32 map over a contiguous [planes][rows][cols] accumulator, box 32 x
// box_rows, 128-byte swizzle (used for TMA reduce-add of dQ tiles).
inline int make_map_f32_acc(CUtensorMap* m, float* base, int rows, int planes, int cols = 64, int box_rows = 128) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is unavailable");
    return POLY_ECUDA;
  }
  const cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)planes};
  const cuuint64_t strides[2] = {(cuuint64_t)cols * 4, (cuuint64_t)rows * cols * 4};
  const cuuint32_t box[3] = {32, (cuuint32_t)box_rows, 1};
  const cuuint32_t es[3] = {1, 1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (dq accumulator) failed (" + std::to_string((int)r) + ")");
    return POLY_ECUDA;
  }
  return POLY_OK;
}

inline bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

// Strides usable by TMA / 16-byte vector access: positive multiples of 8
// elements (16 bytes for 16-bit types).
inline bool strides_ok(const int64_t* st, int n) {
  for (int i = 0; i < n; ++i)
    if (st[i] <= 0 || (st[i] & 7)) return false;
  return true;
}


}  // namespace poly
