// Host-side encoding of TMA tensor maps through the driver entry point
// (looked up once through the runtime, so no direct libcuda symbol is needed).
#include <cudaTypedefs.h>

#include <mutex>

#include "sd_tma.cuh"

namespace sd {

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

static void lookup_encode() {
  void *fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
}

int encode_rows_map(CUtensorMap *map, const void *base, int dtype, int64_t D, int64_t T, int64_t H, int64_t B,
                    int64_t st, int64_t sh, int64_t sb, int box_rows) {
  std::call_once(g_encode_once, lookup_encode);
  if (!g_encode) return SD_ERR_CUDA;
  if (dtype != SD_DTYPE_BF16 && dtype != SD_DTYPE_F16) return SD_ERR_UNSUPPORTED;
  if (D * 2 != 128) return SD_ERR_UNSUPPORTED;
  if (!aligned16(base) || (st * 2) % 16 || (sh * 2) % 16 || (sb * 2) % 16) return SD_ERR_ALIGN;
  const CUtensorMapDataType dt =
      dtype == SD_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(T), static_cast<cuuint64_t>(H),
                        static_cast<cuuint64_t>(B)};
  // strides of dims 1..3 in bytes; a stride may exceed the next dim's extent
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(st * 2), static_cast<cuuint64_t>(sh * 2),
                           static_cast<cuuint64_t>(sb * 2)};
  cuuint32_t box[4] = {static_cast<cuuint32_t>(D), static_cast<cuuint32_t>(box_rows), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = g_encode(map, dt, 4, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SD_OK : SD_ERR_INVALID;
}

int encode_matrix_map(CUtensorMap *map, const void *base, int dtype, int64_t rows, int64_t cols, int64_t ld,
                      int box_rows) {
  std::call_once(g_encode_once, lookup_encode);
  if (!g_encode) return SD_ERR_CUDA;
  if (dtype != SD_DTYPE_BF16 && dtype != SD_DTYPE_F16) return SD_ERR_UNSUPPORTED;
  if (cols % 64 || box_rows < 1 || box_rows > 256) return SD_ERR_UNSUPPORTED;
  if (!aligned16(base) || (ld * 2) % 16) return SD_ERR_ALIGN;
  const CUtensorMapDataType dt =
      dtype == SD_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dt, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SD_OK : SD_ERR_INVALID;
}

int encode_plain_map(CUtensorMap *map, const void *base, int dtype, int64_t rows, int64_t cols, int64_t ld,
                     int box_cols, int box_rows) {
  std::call_once(g_encode_once, lookup_encode);
  if (!g_encode) return SD_ERR_CUDA;
  if (dtype != SD_DTYPE_BF16 && dtype != SD_DTYPE_F16) return SD_ERR_UNSUPPORTED;
  if (box_cols < 8 || box_cols > 256 || box_cols % 8 || box_rows < 1 || box_rows > 256) return SD_ERR_UNSUPPORTED;
  if (!aligned16(base) || (ld * 2) % 16) return SD_ERR_ALIGN;
  const CUtensorMapDataType dt =
      dtype == SD_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dt, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SD_OK : SD_ERR_INVALID;
}

}  // namespace sd
