// Tensor-map TMA shared by the GEMV and the tcgen05 GEMM: 2-D tiled loads completed on mbarriers,
// device-side retargeting of a tensor map to one record, and the host-side encoders of the maps.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace moeb200 {

// 2-D tiled load of box (x, y) of `tmap` into shared memory at `dst`, completing its bytes on `bar`.
// x is in elements of the map's type and must give a 16-byte aligned start.
__device__ __forceinline__ void tma2d(uint32_t dst, uint64_t tmap, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(dst),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// One warp points a global tensor-map slot at a record: the template is staged in shared memory
// (128 bytes at sdesc), its global address replaced, and the result copied out with a release
// fence for the tensor-map proxy; lane 0 then acquires it before issuing loads through it.
__device__ __forceinline__ void retarget_tmap(const CUtensorMap& tmpl, uint32_t sdesc, uint64_t gdesc,
                                              const void* base, int lane) {
  const uint32_t v = reinterpret_cast<const uint32_t*>(&tmpl)[lane];
  asm volatile("st.shared.u32 [%0], %1;" ::"r"(sdesc + 4 * lane), "r"(v) : "memory");
  __syncwarp();
  if (lane == 0)
    asm volatile("tensormap.replace.tile.global_address.shared::cta.b1024.b64 [%0], %1;" ::"r"(sdesc),
                 "l"(reinterpret_cast<uint64_t>(base))
                 : "memory");
  __syncwarp();
  asm volatile("tensormap.cp_fenceproxy.global.shared::cta.tensormap::generic.release.gpu.sync.aligned [%0], [%1], 128;" ::
                   "l"(gdesc),
               "r"(sdesc)
               : "memory");
  if (lane == 0) asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(gdesc) : "memory");
  __syncwarp();
}

// Row maps: a 2-D map of all memory from a base on (rows of rowb bytes) reads every record that lies
// on a multiple of rowb above the base through the row coordinate. They cover kRowMapSpan bytes (every
// record of a process lies well within) and at most 2^31 - 1 rows (int32 coordinates).
constexpr int64_t kRowMapSpan = 1ll << 40;
__host__ __device__ inline int64_t row_map_rows(int64_t rowb) {
  return kRowMapSpan / rowb < 0x7fffffffll ? kRowMapSpan / rowb : 0x7fffffffll;
}
// First row of a field at q in a row map with rows of rowb bytes above base (nrows of the field must
// fit), or -1 for a field that is not on a row of the map.
__device__ __forceinline__ int row_map_first(int64_t q, int64_t base, int64_t rowb, int64_t nrows) {
  const int64_t dq = q - base;
  if (dq < 0) return -1;
  int64_t r, rows;
  if ((rowb & (rowb - 1)) == 0) {  // a power-of-two pitch (every pitch dividing 4096): shifts, no divisions
    const int sh = __ffsll(rowb) - 1;
    if (dq & (rowb - 1)) return -1;
    r = dq >> sh;
    rows = (kRowMapSpan >> sh) < 0x7fffffffll ? (kRowMapSpan >> sh) : 0x7fffffffll;
  } else {
    if (dq % rowb) return -1;
    r = dq / rowb;
    rows = row_map_rows(rowb);
  }
  return r + nrows <= rows ? (int)r : -1;
}

// Host: tensor-map template of a weight field, uint8 [rows][row_bytes] read in boxes of 128 bytes x
// box_rows with 128-byte swizzle. The address is a placeholder (16-byte aligned device memory): the
// kernels swap in each record's address. Cached per shape.
cudaError_t tma_weight_template(CUtensorMap* out, int row_bytes, int rows, int box_rows, void* placeholder);

// Host: 3-D uint8 tensor map [segment][row][128 bytes] of all memory from `base` on: rows of
// row_bytes (a multiple of 128), boxes of box_rows rows x every 128-byte segment of a row, laid out
// segment-major in shared memory with 128-byte swizzle. Cached per (base, row_bytes, box_rows).
cudaError_t tma_rows3d_map(CUtensorMap* out, uint64_t base, int row_bytes, int box_rows);

// Host: 2-D uint8 tensor map [rows][row_bytes] of the memory from `base` on (row_bytes a multiple of
// 128), boxes of 128 bytes x box_rows rows with 128-byte swizzle. Records that lie on row_bytes
// multiples above `base` are read through the row coordinate, so no map is built per record. Cached
// per (base, row_bytes, rows, box_rows).
cudaError_t tma_rows2d_map(CUtensorMap* out, uint64_t base, int row_bytes, int64_t rows, int box_rows);

// Host: tensor map of a row-major 16-bit matrix [rows][cols] at `base`, boxes of 64 columns x
// box_rows with 128-byte swizzle (the K-major operand layout of the tensor cores).
cudaError_t tma_rows16_map(CUtensorMap* out, const void* base, int cols, int rows, int box_rows, int act_type);

}  // namespace moeb200
