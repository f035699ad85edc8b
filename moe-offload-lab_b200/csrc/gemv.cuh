// Grouped expert GEMV ("decode path") and shared work-item declarations.
#pragma once

#include "common.cuh"

namespace moeb200 {

// One unit of grouped work: up to 8*NB (GEMV) or 128 (GEMM) routed pairs that share one
// (expert, precision slot). Field addresses are resolved by whoever builds the list.
struct Item {
  int64_t p_guq;  // gate_up.q (float records: gate_up)
  int64_t p_gus;  // gate_up.s (float records: unused)
  int64_t p_dnq;  // down.q    (float records: down)
  int64_t p_dns;  // down.s
  int32_t slot;   // precision slot (index into GemvParams::lay)
  int32_t start;  // first index into the sorted pair list (and first h row)
  int32_t ntok;   // pairs of this item
  int32_t _pad;
};
static_assert(sizeof(Item) == 48, "Item layout");

struct LayoutDev {
  int32_t wtype;  // MOEB200_F32/F16/BF16/I8/I4
  int32_t gs_up;
  int32_t gs_dn;
  int32_t _pad;
};

struct GemvParams {
  const Item* items;
  const int32_t* n_items;  // device-resident item count
  const int32_t* pos;      // sorted pair list: flat positions t*k + j
  const float* wflat;      // [T*k] router weights
  int32_t k;
  int32_t H;
  int32_t I;
  int32_t T;
  const void* x;   // [T, H] activations
  void* h;         // [n_pairs, I] activations, row j = sorted pair j (unsplit up phase)
  float* pre;      // [n_pairs, 2I] fp32 gate|up pre-activations (split-K up phase), else null
  int32_t* tile_cnt;  // [items, I/16] arrivals of the K splits of each up tile (split-K), zeroed per call
  float* acc;      // [T, H] fp32 combine buffer
  int32_t* status;
  LayoutDev lay[4];
  int32_t ksplit_up;    // K splits of the up phase (1 = write h directly)
  int32_t ksplit_dn;    // K splits of the down phase
  int32_t stage_bytes;  // bytes of one warp stage (32 padded row segments)
  int32_t zero_acc;     // up phase: zero acc before use
};

// Geometry shared by host and device.
constexpr int kGemvStages = 2;
constexpr int kGemvMaxWarps = 12;
constexpr int kStepBytes = 256;  // bytes of one weight row per pipeline step
constexpr int kSplitCols = 512;  // K splits are multiples of this many columns

// Padded stride of one 256-byte row segment in a stage, per record element type: fragment reads of
// the eight rows a warp touches at once then fall in different banks.
__host__ __device__ inline int gemv_row_stride(int wtype) {
  return wtype == MOEB200_I4 ? 288 : wtype == MOEB200_I8 ? 320 : 272;
}

__host__ __device__ inline int gemv_smem_bytes(int stage_bytes, int warps) {
  return warps * (kGemvStages * stage_bytes + kGemvStages * 8);
}

// host launchers (gemv.cu)
cudaError_t launch_gemv_up(const GemvParams& p, int act_type, int nb, int grid, int warps, cudaStream_t s);
cudaError_t launch_gemv_down(const GemvParams& p, int act_type, int nb, int grid, int warps, cudaStream_t s);
cudaError_t launch_finalize(const float* acc, void* out, int act_type, int64_t n, int add, cudaStream_t s);
cudaError_t launch_combine_parts(const float* parts, int G, int64_t n, int act_type, void* out, int add,
                                 cudaStream_t s);
int gemv_occupancy(int act_type, int nb, bool up, bool split, int smem, int warps);
// tcgen05 grouped GEMM (gemm_tc.cu): items of up to 128 pairs, I and H multiples of 128
cudaError_t launch_gemm_up(const GemvParams& p, int act_type, int grid, cudaStream_t s);
cudaError_t launch_gemm_down(const GemvParams& p, int act_type, int grid, cudaStream_t s);

}  // namespace moeb200
