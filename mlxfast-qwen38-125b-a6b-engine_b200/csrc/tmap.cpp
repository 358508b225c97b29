// tmap.cpp -- TMA tensor-map encoding through the driver entry point
// (cudaGetDriverEntryPoint, so the library needs no link-time libcuda).
#include "tmap.hpp"

#include <cudaTypedefs.h>

#include <mutex>

#include "host.hpp"

namespace b2q {

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int make_row_block_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t row_bytes, uint32_t box_bytes,
                       bool swizzled) {
  auto fn = encode_fn();
  if (!fn) return set_error(B2Q_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r;
  if (swizzled) {
    if (row_bytes % 128 || box_bytes % 128 || box_bytes / 128 > 256)
      return set_error(B2Q_EINVAL, "tensor map: swizzled rows need 128-byte pieces (row %llu, box %u)",
                       (unsigned long long)row_bytes, box_bytes);
    cuuint64_t dims[3] = {64, rows, row_bytes / 128};
    cuuint64_t strides[2] = {row_bytes, 128};
    cuuint32_t box[3] = {64, 8, box_bytes / 128};
    r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(base), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    if (row_bytes % 16 || box_bytes % 16 || box_bytes / 2 > 256)
      return set_error(B2Q_EINVAL, "tensor map: rows of %llu bytes / box of %u bytes not in 16-byte units",
                       (unsigned long long)row_bytes, box_bytes);
    cuuint64_t dims[2] = {row_bytes / 2, rows};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_bytes / 2, 8};
    r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS)
    return set_error(B2Q_ECUDA, "cuTensorMapEncodeTiled failed (%d) for rows=%llu row_bytes=%llu box=%u", (int)r,
                     (unsigned long long)rows, (unsigned long long)row_bytes, box_bytes);
  return B2Q_OK;
}

int make_row_tile_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t row_bytes, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return set_error(B2Q_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (row_bytes % 128 || row_bytes / 128 > 256 || box_rows < 1 || box_rows > 256 || rows < box_rows ||
      (reinterpret_cast<uintptr_t>(base) & 15))
    return set_error(B2Q_EINVAL, "tensor map: rows of %llu bytes in boxes of %u rows not encodable",
                     (unsigned long long)row_bytes, box_rows);
  cuuint64_t dims[3] = {64, rows, row_bytes / 128};
  cuuint64_t strides[2] = {row_bytes, 128};
  cuuint32_t box[3] = {64, box_rows, (cuuint32_t)(row_bytes / 128)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(B2Q_ECUDA, "cuTensorMapEncodeTiled failed (%d) for rows=%llu row_bytes=%llu box_rows=%u", (int)r,
                     (unsigned long long)rows, (unsigned long long)row_bytes, box_rows);
  return B2Q_OK;
}

int make_2d_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t row_bytes, uint32_t box_bytes,
                uint32_t box_rows, int swizzle_bytes) {
  auto fn = encode_fn();
  if (!fn) return set_error(B2Q_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  CUtensorMapSwizzle sw;
  switch (swizzle_bytes) {
    case 0: sw = CU_TENSOR_MAP_SWIZZLE_NONE; break;
    case 32: sw = CU_TENSOR_MAP_SWIZZLE_32B; break;
    case 64: sw = CU_TENSOR_MAP_SWIZZLE_64B; break;
    case 128: sw = CU_TENSOR_MAP_SWIZZLE_128B; break;
    default: return set_error(B2Q_EINVAL, "tensor map: swizzle of %d bytes", swizzle_bytes);
  }
  if (row_bytes % 16 || box_bytes % 16 || box_bytes / 2 > 256 || box_rows < 1 || box_rows > 256 ||
      (swizzle_bytes && box_bytes > (uint32_t)swizzle_bytes) || (reinterpret_cast<uintptr_t>(base) & 15))
    return set_error(B2Q_EINVAL, "tensor map: rows of %llu bytes, box %u x %u, swizzle %d not encodable",
                     (unsigned long long)row_bytes, box_bytes, box_rows, swizzle_bytes);
  cuuint64_t dims[2] = {row_bytes / 2, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_bytes / 2, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(B2Q_ECUDA, "cuTensorMapEncodeTiled failed (%d) for rows=%llu row_bytes=%llu box=%ux%u", (int)r,
                     (unsigned long long)rows, (unsigned long long)row_bytes, box_bytes, box_rows);
  return B2Q_OK;
}

}  // namespace b2q
