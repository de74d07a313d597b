// Host-side creation of TMA tensor maps through the driver entry point
// (no link-time dependency on libcuda).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace llmyb {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = []() -> PFN_cuTensorMapEncodeTiled_v12000 {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// Row-major bf16 matrix [rows, cols] (row stride ld elements) tiled into boxes
// of [box_rows, box_cols] with the 128-byte swizzle; box_cols * 2 must be 128.
inline bool make_bf16_2d_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                             uint64_t ld, uint32_t box_rows, uint32_t box_cols) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (ld * 2) % 16 != 0) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Token-major bf16 tensor [batch][rows][cols] (row stride ld elements, batch
// stride rows * ld) tiled into boxes of [1, box_rows, 64 cols] with the
// 128-byte swizzle.  Rows past `rows` read as zeros, so a box never crosses
// into the next batch entry.
inline bool make_bf16_3d_map(CUtensorMap* map, const void* base, uint64_t batch, uint64_t rows,
                             uint64_t cols, uint64_t ld, uint32_t box_rows) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (ld * 2) % 16 != 0) return false;
  cuuint64_t dims[3] = {cols, rows, batch};
  cuuint64_t strides[2] = {ld * 2, rows * ld * 2};
  cuuint32_t box[3] = {64, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Packed bf16 tensor [batch][rows][heads][cols] tiled into boxes of
// [1, box_rows, 1, 64 cols] with the 128-byte swizzle (one head, box_rows
// consecutive rows; rows past `rows` read as zeros).
inline bool make_bf16_4d_map(CUtensorMap* map, const void* base, uint64_t batch, uint64_t rows,
                             uint64_t heads, uint64_t cols, uint32_t box_rows) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (cols * 2) % 16 != 0) return false;
  cuuint64_t dims[4] = {cols, heads, rows, batch};
  cuuint64_t strides[3] = {cols * 2, heads * cols * 2, rows * heads * cols * 2};
  cuuint32_t box[4] = {64, 1, box_rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// bf16 tensor [batch][rows][heads][cols] with row stride ld elements (a head
// slice of a wider token-major row), boxes of [1, box_rows, 1, 64 cols] with
// the 128-byte swizzle; rows past `rows` and columns past `cols` read as zeros.
inline bool make_bf16_4d_map_ld(CUtensorMap* map, const void* base, uint64_t batch,
                                uint64_t rows, uint64_t heads, uint64_t cols, uint64_t ld,
                                uint32_t box_rows) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (cols * 2) % 16 != 0 || (ld * 2) % 16 != 0)
    return false;
  cuuint64_t dims[4] = {cols, heads, rows, batch};
  cuuint64_t strides[3] = {cols * 2, ld * 2, rows * ld * 2};
  cuuint32_t box[4] = {64, 1, box_rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// SMs of the current device (queried on every call: the attribute belongs to
// the device, and the query is cheap).
inline int num_sms() {
  int dev = 0, v = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
  return v > 0 ? v : 148;
}

}  // namespace llmyb
