// Host-side TMA descriptor construction shared by the sm_100a kernels. cuTensorMapEncodeTiled is
// fetched from the driver at run time (cudaGetDriverEntryPoint), so the library does not link
// against libcuda and loads on machines without a GPU.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "fea_params.h"

namespace vmb {
namespace tma {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
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

// 5-D map over the view `v` of a [batch][rows][cols] tensor (fea_params.h): dims (cols, rows, n1,
// n2, batch / (n1 n2)), so a tile of batch entry s is addressed as (x, y, s % n1, s / n1 % n2,
// s / (n1 n2)). Boxes of `box_cols` columns (128 B, one swizzle row) x `box_rows` rows, 128-byte
// swizzle. Rows past `rows` read as zeros and are clipped on stores, per batch entry. Strides must
// be multiples of 16 bytes (token-major head strides of D * 2 bytes are); the stride of an extent-1
// dimension is never used and is replaced by a valid value.
inline bool make_map5(CUtensorMap* m, CUtensorMapDataType dt, int esize, const void* base, int64_t cols, int64_t rows,
                      int64_t batch, const View& v, int n1, int n2, int box_cols, int box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc || n1 < 1 || n2 < 1 || batch < 1 || batch % ((int64_t)n1 * n2)) return false;
  const int64_t n3 = batch / ((int64_t)n1 * n2);
  const int64_t ext[4] = {rows, n1, n2, n3};
  const int64_t str[4] = {v.rs, v.s1, v.s2, v.s3};
  cuuint64_t dims[5] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)n1, (cuuint64_t)n2, (cuuint64_t)n3};
  cuuint64_t strides[4];
  for (int i = 0; i < 4; ++i) {
    int64_t bytes = str[i] * esize;
    if (ext[i] == 1 && (bytes <= 0 || bytes % 16)) bytes = v.rs * esize * (rows > 0 ? rows : 1);
    if (bytes <= 0 || bytes % 16) return false;
    strides[i] = (cuuint64_t)bytes;
  }
  cuuint32_t box[5] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows, 1, 1, 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  return enc(m, dt, 5, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 16-bit elements, boxes of 64 columns.
inline bool make_map_view(CUtensorMap* m, const void* base, bool bf16, int64_t cols, int64_t rows, int64_t batch,
                          const View& v, int n1, int n2, int box_rows) {
  return make_map5(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, cols, rows,
                   batch, v, n1, n2, 64, box_rows);
}

// e4m3 (one-byte) elements, boxes of 128 columns.
inline bool make_map_view_e4m3(CUtensorMap* m, const void* base, int64_t cols, int64_t rows, int64_t batch,
                               const View& v, int n1, int n2, int box_rows) {
  return make_map5(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, base, cols, rows, batch, v, n1, n2, 128, box_rows);
}

// fp32 elements, boxes of 32 columns.
inline bool make_map_view_f32(CUtensorMap* m, const void* base, int64_t cols, int64_t rows, int64_t batch,
                              const View& v, int n1, int n2, int box_rows) {
  return make_map5(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, cols, rows, batch, v, n1, n2, 32, box_rows);
}

// Dense [batch][rows][cols] with batch stride `bs` elements (internal buffers), split (n1, n2).
inline bool make_map(CUtensorMap* m, const void* base, bool bf16, int64_t cols, int64_t rows, int64_t batch,
                     int64_t bs, int box_rows, int n1 = 1, int n2 = 1) {
  return make_map_view(m, base, bf16, cols, rows, batch, dense_view(cols, bs, n1, n2), n1, n2, box_rows);
}
inline bool make_map_f32(CUtensorMap* m, const void* base, int64_t cols, int64_t rows, int64_t batch, int64_t bs,
                         int box_rows, int n1 = 1, int n2 = 1) {
  return make_map_view_f32(m, base, cols, rows, batch, dense_view(cols, bs, n1, n2), n1, n2, box_rows);
}

}  // namespace tma
}  // namespace vmb
