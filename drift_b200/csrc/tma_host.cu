// Tensor maps for the TMA copies (tma_host.cuh).
#include <cuda.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "tma_host.cuh"

namespace drift {

namespace {

typedef CUresult (*EncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled lookup_encode_tiled() {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
          cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    return reinterpret_cast<EncodeTiled>(p);
  return nullptr;
}

// Looked up once per process; a function-local static is initialised by one
// thread while any other first caller waits, so no caller sees it half made.
EncodeTiled encode_tiled() {
  static const EncodeTiled fn = lookup_encode_tiled();
  return fn;
}

}  // namespace

bool tensor_maps_available() { return encode_tiled() != nullptr; }

int encode_word_rows(CUtensorMap* map, const void* base, int64_t row_words, int64_t rows,
                     int box_words, int box_rows) {
  EncodeTiled encode = encode_tiled();
  if (!encode) return invalid("cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[2] = {cuuint64_t(row_words), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(row_words * 4)};
  const cuuint32_t box[2] = {cuuint32_t(box_words), cuuint32_t(box_rows)};
  const cuuint32_t element[2] = {1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(base), dims,
                            strides, box, element, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return invalid("weight tensor map refused (CUresult %d)", int(r));
  return 0;
}

int encode_f16_sw128(CUtensorMap* map, const void* base, int64_t cols, int64_t rows, int box_rows) {
  EncodeTiled encode = encode_tiled();
  if (!encode) return invalid("cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(cols * 2)};
  const cuuint32_t box[2] = {64, cuuint32_t(box_rows)};
  const cuuint32_t element[2] = {1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims,
                            strides, box, element, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return invalid("x tensor map refused (CUresult %d)", int(r));
  return 0;
}

}  // namespace drift
