// Expert-parallel exchange rows (no moelab counterpart: moelab runs on one GPU).
//
// Under expert parallelism every rank routes its own tokens and then needs, on the ranks owning
// the chosen experts, each token's hidden row together with its routing (top-k indices, weights,
// precision levels, skip flags). One token travels as one fixed-size row
//
//   [ x: H act-type values | idx: k int64 | w: k float32 | level: k uint8 | skip: k uint8 | pad to 16 B ]
//
// so a whole rank's tokens move in one collective (or one peer copy), and the receiver splits the
// gathered rows back into the contiguous arrays the expert kernels read.
#include "common.cuh"

#include <cstdarg>
#include <cstdio>

namespace moeb200 {
int set_error(int code, const char* fmt, ...);
}

namespace {

using namespace moeb200;

int elem_bytes(int act) { return act == MOEB200_F32 ? 4 : 2; }

size_t row_bytes(int H, int k, int act) {
  const size_t b = (size_t)H * elem_bytes(act) + (size_t)k * 14;
  return (b + 15) / 16 * 16;
}

// One block per token row; x moves as 16-byte vectors, the routing bytes one per thread.
__global__ void ep_pack_kernel(const uint8_t* __restrict__ x, const int64_t* __restrict__ idx,
                               const float* __restrict__ w, const uint8_t* __restrict__ level,
                               const uint8_t* __restrict__ skip, int xbytes, int k, int rb, uint8_t* __restrict__ rows) {
  const int t = blockIdx.x;
  uint8_t* row = rows + (int64_t)t * rb;
  const uint4* xs = reinterpret_cast<const uint4*>(x + (int64_t)t * xbytes);
  uint4* xd = reinterpret_cast<uint4*>(row);
  for (int i = threadIdx.x; i < xbytes / 16; i += blockDim.x) xd[i] = xs[i];
  int64_t* ri = reinterpret_cast<int64_t*>(row + xbytes);
  float* rw = reinterpret_cast<float*>(row + xbytes + 8 * k);
  uint8_t* rl = row + xbytes + 12 * k;
  uint8_t* rs = rl + k;
  for (int j = threadIdx.x; j < k; j += blockDim.x) {
    const int64_t p = (int64_t)t * k + j;
    ri[j] = idx[p];
    rw[j] = w[p];
    rl[j] = level ? level[p] : 0;
    rs[j] = skip ? skip[p] : 0;
  }
  for (int j = xbytes + 14 * k + threadIdx.x; j < rb; j += blockDim.x) row[j] = 0;
}

__global__ void ep_unpack_kernel(const uint8_t* __restrict__ rows, int xbytes, int k, int rb, uint8_t* __restrict__ x,
                                 int64_t* __restrict__ idx, float* __restrict__ w, uint8_t* __restrict__ level,
                                 uint8_t* __restrict__ skip) {
  const int t = blockIdx.x;
  const uint8_t* row = rows + (int64_t)t * rb;
  if (x) {
    const uint4* xs = reinterpret_cast<const uint4*>(row);
    uint4* xd = reinterpret_cast<uint4*>(x + (int64_t)t * xbytes);
    for (int i = threadIdx.x; i < xbytes / 16; i += blockDim.x) xd[i] = xs[i];
  }
  const int64_t* ri = reinterpret_cast<const int64_t*>(row + xbytes);
  const float* rw = reinterpret_cast<const float*>(row + xbytes + 8 * k);
  const uint8_t* rl = row + xbytes + 12 * k;
  const uint8_t* rs = rl + k;
  for (int j = threadIdx.x; j < k; j += blockDim.x) {
    const int64_t p = (int64_t)t * k + j;
    idx[p] = ri[j];
    w[p] = rw[j];
    if (level) level[p] = rl[j];
    if (skip) skip[p] = rs[j];
  }
}

int check_args(int n, int H, int k, int act, const char* who) {
  if (n <= 0 || H <= 0 || k <= 0 || k > 32)
    return set_error(MOEB200_ERR_INVALID, "%s: bad sizes n=%d H=%d k=%d", who, n, H, k);
  if (act != MOEB200_F16 && act != MOEB200_BF16 && act != MOEB200_F32)
    return set_error(MOEB200_ERR_UNSUPPORTED, "%s: activations must be F32, F16 or BF16", who);
  if (((size_t)H * elem_bytes(act)) % 16)
    return set_error(MOEB200_ERR_UNSUPPORTED, "%s: a hidden row must be a multiple of 16 bytes", who);
  return MOEB200_OK;
}

}  // namespace

extern "C" {

size_t moeb200_ep_row_bytes(int32_t H, int32_t k, int32_t act_type) {
  if (H <= 0 || k <= 0) return 0;
  return row_bytes(H, k, act_type);
}

int moeb200_ep_pack(const void* x, const int64_t* idx, const float* w, const uint8_t* level, const uint8_t* skip,
                    int32_t T, int32_t H, int32_t k, int32_t act_type, void* rows, void* stream) {
  if (!x || !idx || !w || !rows) return set_error(MOEB200_ERR_INVALID, "ep_pack: null pointer");
  int rc = check_args(T, H, k, act_type, "ep_pack");
  if (rc) return rc;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(rows)) % 16)
    return set_error(MOEB200_ERR_INVALID, "ep_pack: x and rows must be 16-byte aligned");
  const int xb = H * elem_bytes(act_type);
  ep_pack_kernel<<<T, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(x), idx, w, level, skip, xb, k, (int)row_bytes(H, k, act_type),
      static_cast<uint8_t*>(rows));
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(MOEB200_ERR_CUDA, "ep_pack: %s", cudaGetErrorString(e));
  return MOEB200_OK;
}

int moeb200_ep_unpack(const void* rows, int32_t n, int32_t H, int32_t k, int32_t act_type, void* x, int64_t* idx,
                      float* w, uint8_t* level, uint8_t* skip, void* stream) {
  if (!rows || !idx || !w) return set_error(MOEB200_ERR_INVALID, "ep_unpack: null pointer");
  int rc = check_args(n, H, k, act_type, "ep_unpack");
  if (rc) return rc;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(rows)) % 16)
    return set_error(MOEB200_ERR_INVALID, "ep_unpack: x and rows must be 16-byte aligned");
  const int xb = H * elem_bytes(act_type);
  ep_unpack_kernel<<<n, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(rows), xb, k, (int)row_bytes(H, k, act_type), static_cast<uint8_t*>(x), idx, w, level,
      skip);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(MOEB200_ERR_CUDA, "ep_unpack: %s", cudaGetErrorString(e));
  return MOEB200_OK;
}

}  // extern "C"
