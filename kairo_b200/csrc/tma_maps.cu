// Host-side TMA tensor maps of the tcgen05 SpMM kernels.
//
// cuTensorMapEncodeTiled is a driver API; it is resolved once through the
// runtime's driver entry-point query so that the library links against the
// CUDA runtime only.
#include <cuda.h>

#include <mutex>
#include <sstream>

#include "internal.h"

namespace kairo {
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

CUtensorMapSwizzle swizzle_for_bytes(int inner_bytes) {
  return inner_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
         : inner_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                             : CU_TENSOR_MAP_SWIZZLE_32B;
}

}  // namespace

kairo_status make_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes,
                         uint64_t inner, uint64_t outer, uint64_t row_stride_elems, uint32_t box_inner,
                         uint32_t box_outer, const char* what) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(KAIRO_STATUS_CUDA_ERROR, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_stride_elems * static_cast<uint64_t>(elem_bytes)};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle_for_bytes(static_cast<int>(box_inner) * elem_bytes), CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    std::ostringstream os;
    os << "cuTensorMapEncodeTiled failed for " << what << " (CUresult " << static_cast<int>(r) << ")";
    return fail(KAIRO_STATUS_INVALID_VALUE, os.str());
  }
  return KAIRO_STATUS_SUCCESS;
}

kairo_status make_map_b3d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t n, uint64_t k,
                          uint64_t ldb, uint32_t bk, uint32_t atoms) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(KAIRO_STATUS_CUDA_ERROR, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[3] = {64, k, n / 64};
  const cuuint64_t strides[2] = {ldb * 2, 128};
  const cuuint32_t box[3] = {64, bk, atoms};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    std::ostringstream os;
    os << "cuTensorMapEncodeTiled failed for the 3D view of B (CUresult " << static_cast<int>(r) << ")";
    return fail(KAIRO_STATUS_INVALID_VALUE, os.str());
  }
  return KAIRO_STATUS_SUCCESS;
}

kairo_status make_block_run_map(const kairo_bsr* a, int blocks, CUtensorMap* map) {
  const CUtensorMapDataType dt =
      a->dtype == KAIRO_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  return make_map_2d(map, a->blocks, dt, 2, static_cast<uint64_t>(a->bk),
                     static_cast<uint64_t>(a->nblocks_stored) * a->bm, static_cast<uint64_t>(a->bk),
                     static_cast<uint32_t>(a->bk), static_cast<uint32_t>(blocks * a->bm), "runs of block storage");
}

kairo_status make_operand_maps(const kairo_bsr* a, const void* b, int64_t ldb, bool linear, int64_t n, int nt,
                               CUtensorMap* map_a, CUtensorMap* map_b, int* b_box3d) {
  const CUtensorMapDataType dt =
      a->dtype == KAIRO_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  kairo_status st = make_map_2d(map_a, a->blocks, dt, 2, static_cast<uint64_t>(a->bk),
                                static_cast<uint64_t>(a->nblocks_stored) * a->bm, static_cast<uint64_t>(a->bk),
                                static_cast<uint32_t>(a->bk), static_cast<uint32_t>(a->bm), "block storage");
  if (st) return st;
  *b_box3d = 0;
  if (!linear) {
    if (n % 64 == 0) {
      st = make_map_b3d(map_b, b, dt, static_cast<uint64_t>(n), static_cast<uint64_t>(a->cols),
                        static_cast<uint64_t>(ldb), static_cast<uint32_t>(a->bk), static_cast<uint32_t>(2 * nt));
      *b_box3d = (st == KAIRO_STATUS_SUCCESS);
    }
    if (!*b_box3d)
      st = make_map_2d(map_b, b, dt, 2, static_cast<uint64_t>(n), static_cast<uint64_t>(a->cols),
                       static_cast<uint64_t>(ldb), 64, static_cast<uint32_t>(a->bk), "B");
  } else {
    st = make_map_2d(map_b, b, dt, 2, static_cast<uint64_t>(a->cols), static_cast<uint64_t>(n),
                     static_cast<uint64_t>(ldb), static_cast<uint32_t>(a->bk), static_cast<uint32_t>(128 * nt), "X");
  }
  return st;
}

}  // namespace kairo
