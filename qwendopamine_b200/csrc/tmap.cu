// tmap.cu -- host-side TMA tensor maps (cuTensorMapEncodeTiled, reached
// through the runtime's driver entry point so the library needs no link
// against libcuda).  Declared in tc.cuh.
#include <cuda.h>
#include <cuda_runtime.h>

#include "tc.cuh"

namespace gdn2 {
namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

}  // namespace

bool tmap_available() { return encode_fn() != nullptr; }

bool tmap_2d_bf16(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint32_t box_x,
                  bool swizzle) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {inner * 2};
  cuuint32_t box[2] = {box_x, 64};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool tmap_2d_box_bf16(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows,
                      uint32_t box_x, uint32_t box_y) {
  EncodeTiledFn enc = encode_fn();
  if (!enc || box_x * 2 != 128 || box_y == 0 || box_y > 256) return false;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {inner * 2};
  cuuint32_t box[2] = {box_x, box_y};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool tmap_rows(CUtensorMap* m, const void* base, uint64_t D, uint64_t H, uint64_t rows,
               uint32_t box_x, int elem_bytes) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  if (box_x * (uint32_t)elem_bytes != 128) return false;  // one 128-byte swizzle span
  cuuint64_t dims[3] = {D, H, rows};
  cuuint64_t strides[2] = {D * (uint64_t)elem_bytes, H * D * (uint64_t)elem_bytes};
  cuuint32_t box[3] = {box_x, 1, 64};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
             3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool tmap_plain(CUtensorMap* m, const void* base, int rank, const uint64_t* dims,
                const uint64_t* strides_bytes, const uint32_t* box, int elem_bytes) {
  EncodeTiledFn enc = encode_fn();
  if (!enc || rank < 2 || rank > 3) return false;
  cuuint64_t d[3], st[2];
  cuuint32_t bx[3], estr[3] = {1, 1, 1};
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    if (i + 1 < rank) st[i] = strides_bytes[i];
  }
  return enc(m, elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
             (cuuint32_t)rank, const_cast<void*>(base), d, st, bx, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace gdn2
