// TMA tensor-map encoding (host). cuTensorMapEncodeTiled is fetched from the driver at run time
// through the runtime's entry-point query, so the library does not link libcuda directly and loads
// on machines without a GPU driver.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "g16_internal.cuh"

namespace g16 {
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn(int* status) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (err == cudaSuccess && q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  if (fn == nullptr) *status = err != cudaSuccess ? cuda_fail(err) : G16_ERR_CUDA;
  return fn;
}

}  // namespace

// 2-D tensor map over a row-major [rows, cols] matrix whose rows are row_stride elements apart,
// with a [box_rows, box_cols] box. Out-of-range box elements read as zero and are not stored.
int make_tmap_2d_strided(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint32_t elem_bytes,
                         uint64_t rows, uint64_t cols, uint64_t row_stride, uint32_t box_rows, uint32_t box_cols,
                         CUtensorMapSwizzle swz) {
  int st = G16_OK;
  auto fn = encode_fn(&st);
  if (fn == nullptr) return st;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {row_stride * elem_bytes};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? G16_OK : G16_ERR_CUDA;
}

// Contiguous rows (row_stride = cols).
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint32_t elem_bytes, uint64_t rows,
                 uint64_t cols, uint32_t box_rows, uint32_t box_cols, CUtensorMapSwizzle swz) {
  return make_tmap_2d_strided(map, base, dt, elem_bytes, rows, cols, cols, box_rows, box_cols, swz);
}

}  // namespace g16
