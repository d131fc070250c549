// rk_tma.h -- host-side construction of 2-D TMA tensor maps (CUtensorMap)
// for row-major 16-bit matrices, with the 128-byte swizzle the UMMA
// shared-memory descriptors expect.  cuTensorMapEncodeTiled is fetched from
// the driver at run time, so the library does not link libcuda directly.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>

#include "rk_internal.h"

namespace rk {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Tensor map over a row-major [outer, inner] matrix of 16-bit elements, read
// in boxes of [box_outer, box_inner] with the 128-byte swizzle
// (box_inner * 2 must be <= 128).  Out-of-range elements read as zero.
inline rk_status encode_tmap_2d(CUtensorMap* map, const void* base, rk_dtype dt, int64_t inner,
                                int64_t outer, uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (fn == nullptr) return RK_ERR_CUDA;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(inner) * 2};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estride[2] = {1, 1};
  const CUtensorMapDataType t =
      dt == RK_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = fn(map, t, 2, const_cast<void*>(base), dims, strides, box, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r == CUDA_SUCCESS) return RK_OK;
  note_error("cuTensorMapEncodeTiled failed (CUresult " + std::to_string(static_cast<int>(r)) +
             ") for a [" + std::to_string(outer) + ", " + std::to_string(inner) + "] matrix at " +
             std::to_string(reinterpret_cast<uintptr_t>(base)) + " with box [" +
             std::to_string(box_outer) + ", " + std::to_string(box_inner) + "]");
  return RK_ERR_UNSUPPORTED;
}

// Tensor map over a stack of `depth` row-major [rows, inner] matrices of 16-bit elements
// (dense: matrix i starts rows * inner elements after matrix i - 1), read in boxes of
// [1, box_rows, box_inner] with the 128-byte swizzle.  Rows past the end of a matrix read
// as zero (no spill into the next matrix).
inline rk_status encode_tmap_3d(CUtensorMap* map, const void* base, rk_dtype dt, int64_t inner,
                                int64_t rows, int64_t depth, uint32_t box_inner,
                                uint32_t box_rows) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (fn == nullptr) return RK_ERR_CUDA;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows),
                              static_cast<cuuint64_t>(depth)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(inner) * 2,
                                 static_cast<cuuint64_t>(inner) * static_cast<cuuint64_t>(rows) * 2};
  const cuuint32_t box[3] = {box_inner, box_rows, 1};
  const cuuint32_t estride[3] = {1, 1, 1};
  const CUtensorMapDataType t =
      dt == RK_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = fn(map, t, 3, const_cast<void*>(base), dims, strides, box, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r == CUDA_SUCCESS) return RK_OK;
  note_error("cuTensorMapEncodeTiled failed (CUresult " + std::to_string(static_cast<int>(r)) +
             ") for a [" + std::to_string(depth) + ", " + std::to_string(rows) + ", " +
             std::to_string(inner) + "] stack");
  return RK_ERR_UNSUPPORTED;
}

// Encoding a tensor map costs about a microsecond of host time per call; decode loops
// call the same GEMV on the same weight and activation buffers every step, so recently
// encoded maps are kept in a small process-wide cache keyed by every encoded field.
struct TmapKey {
  const void* base;
  int64_t inner, outer;
  uint32_t box_inner, box_outer;
  int dt;
  bool operator==(const TmapKey& o) const {
    return base == o.base && inner == o.inner && outer == o.outer && box_inner == o.box_inner &&
           box_outer == o.box_outer && dt == o.dt;
  }
};

inline rk_status make_tmap_2d(CUtensorMap* map, const void* base, rk_dtype dt, int64_t inner,
                              int64_t outer, uint32_t box_inner, uint32_t box_outer) {
  constexpr int kSlots = 64;
  struct Slot {
    TmapKey key;
    CUtensorMap map;
    bool used;
  };
  static Slot slots[kSlots];
  static int next = 0;
  static std::mutex mu;
  const TmapKey key{base, inner, outer, box_inner, box_outer, static_cast<int>(dt)};
  {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < kSlots; ++i)
      if (slots[i].used && slots[i].key == key) {
        *map = slots[i].map;
        return RK_OK;
      }
  }
  const rk_status st = encode_tmap_2d(map, base, dt, inner, outer, box_inner, box_outer);
  if (st != RK_OK) return st;
  std::lock_guard<std::mutex> lock(mu);
  slots[next] = Slot{key, *map, true};
  next = (next + 1) % kSlots;
  return RK_OK;
}

}  // namespace rk
