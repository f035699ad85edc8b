// Host-side tensor-map encoders (cuTensorMapEncodeTiled through the runtime's driver entry point).
#include <cudaTypedefs.h>

#include <map>
#include <mutex>
#include <tuple>

#include "tma.cuh"

namespace moeb200 {

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q{};
    void* fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return encode;
}

}  // namespace

cudaError_t tma_weight_template(CUtensorMap* out, int row_bytes, int rows, int box_rows, void* placeholder) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int>, CUtensorMap> cache;
  std::lock_guard<std::mutex> lk(mu);
  const auto key = std::make_tuple(row_bytes, rows, box_rows);
  auto f = cache.find(key);
  if (f != cache.end()) {
    *out = f->second;
    return cudaSuccess;
  }
  auto encode = encode_fn();
  if (!encode) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  const cuuint32_t box[2] = {128u, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1u, 1u};
  CUtensorMap m;
  const CUresult r = encode(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, placeholder, dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  cache[key] = m;
  *out = m;
  return cudaSuccess;
}

cudaError_t tma_rows3d_map(CUtensorMap* out, uint64_t base, int row_bytes, int box_rows) {
  static std::mutex mu;
  static std::map<std::tuple<uint64_t, int, int>, CUtensorMap> cache;
  std::lock_guard<std::mutex> lk(mu);
  const auto key = std::make_tuple(base, row_bytes, box_rows);
  auto f = cache.find(key);
  if (f != cache.end()) {
    *out = f->second;
    return cudaSuccess;
  }
  auto encode = encode_fn();
  if (!encode) return cudaErrorNotSupported;
  // [segment][row][128 bytes]: dim 0 the bytes of a 128-byte segment, dim 1 rows (pitch row_bytes),
  // dim 2 the row's segments (pitch 128); a box is box_rows rows x every segment, segment-major
  const cuuint64_t dims[3] = {128u, 0x7fffffffull, (cuuint64_t)(row_bytes / 128)};
  const cuuint64_t strides[2] = {(cuuint64_t)row_bytes, 128u};
  const cuuint32_t box[3] = {128u, (cuuint32_t)box_rows, (cuuint32_t)(row_bytes / 128)};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  CUtensorMap m;
  const CUresult r = encode(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, reinterpret_cast<void*>(base), dims, strides, box,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  if (cache.size() > 256) cache.clear();
  cache[key] = m;
  *out = m;
  return cudaSuccess;
}

cudaError_t tma_rows2d_map(CUtensorMap* out, uint64_t base, int row_bytes, int64_t rows, int box_rows) {
  static std::mutex mu;
  static std::map<std::tuple<uint64_t, int, int64_t, int>, CUtensorMap> cache;
  std::lock_guard<std::mutex> lk(mu);
  if (row_bytes < 128 || row_bytes % 128 || box_rows < 1 || box_rows > 256 || rows < box_rows || rows > 0x7fffffffll)
    return cudaErrorInvalidValue;
  const auto key = std::make_tuple(base, row_bytes, rows, box_rows);
  auto f = cache.find(key);
  if (f != cache.end()) {
    *out = f->second;
    return cudaSuccess;
  }
  auto encode = encode_fn();
  if (!encode) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  const cuuint32_t box[2] = {128u, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1u, 1u};
  CUtensorMap m;
  const CUresult r = encode(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, reinterpret_cast<void*>(base), dims, strides, box,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  if (cache.size() > 256) cache.clear();
  cache[key] = m;
  *out = m;
  return cudaSuccess;
}

cudaError_t tma_rows16_map(CUtensorMap* out, const void* base, int cols, int rows, int box_rows, int act_type) {
  auto encode = encode_fn();
  if (!encode) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1u, 1u};
  const CUtensorMapDataType dt =
      act_type == MOEB200_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = encode(out, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace moeb200
