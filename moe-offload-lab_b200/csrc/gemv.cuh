// Grouped expert GEMV ("decode path") shared declarations.
#pragma once

#include "common.cuh"

namespace moeb200 {

// One unit of grouped work: up to 8*NB routed pairs that share one (expert, precision slot).
// Field addresses are resolved by the producer of the list (dispatch or the pointer-table entry).
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
  void* h;         // [n_pairs, I] activations, row j = sorted pair j
  float* acc;      // [T, H] fp32 combine buffer
  int32_t* status;
  LayoutDev lay[4];
  int32_t scale_slot_bytes;  // bytes of one per-tile scale block slot
  int32_t zero_acc;          // up phase: zero acc before use
};

// Launch-time geometry shared by host and device.
constexpr int kGemvStages = 2;
constexpr int kGemvWarps = 6;
constexpr int kStageRowBytes = 192;   // max padded row stride of one stage (int8 layout)
constexpr int kStepBytes = 128;       // bytes of one weight row per pipeline step (<= kStageRowBytes - 64)
constexpr int kStageBytes = 32 * kStageRowBytes;

__host__ __device__ inline int gemv_warp_smem(int scale_slot_bytes) {
  return kGemvStages * kStageBytes + kGemvStages * scale_slot_bytes;
}

// host launchers (gemv.cu)
cudaError_t launch_gemv_up(const GemvParams& p, int act_type, int nb, int grid, cudaStream_t s);
cudaError_t launch_gemv_down(const GemvParams& p, int act_type, int nb, int grid, cudaStream_t s);
cudaError_t launch_finalize(const float* acc, void* out, int act_type, int64_t n, int add, cudaStream_t s);
// tcgen05 grouped GEMM (gemm_tc.cu): items of up to 128 pairs, I and H multiples of 128
cudaError_t launch_gemm_up(const GemvParams& p, int act_type, int grid, cudaStream_t s);
cudaError_t launch_gemm_down(const GemvParams& p, int act_type, int grid, cudaStream_t s);
int gemv_smem_bytes(int scale_slot_bytes);

}  // namespace moeb200
