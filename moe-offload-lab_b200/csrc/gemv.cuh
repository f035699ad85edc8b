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
  void* h;         // [n_pairs, I] activations, row j = sorted pair j
  float* pre;      // [kMaxKSplit][pre_rows][2I] fp32 gate|up pre-activations of each K split (split-K
                   // up phase), else null
  int32_t* tile_cnt;  // [items, I/16] arrivals of the K splits of each up job (split-K), zeroed by the
                      // kernel that wrote the items
  float* acc;      // [T, H] fp32 combine buffer
  int32_t* status;
  LayoutDev lay[4];
  int32_t ksplit_up;    // K splits of the up phase (1 = write h directly)
  int32_t ksplit_dn;    // K splits of the down phase
  void* tmap_ws;        // [4 * grid] 128-byte tensor-map slots of the GEMV CTAs (device memory)
  // shared-memory geometry of a GEMV launch (set by launch_gemv_phases)
  int32_t b_stride;     // bytes between two token rows of a stage
  int32_t b_rows;       // token rows of a stage (8 * NB)
  int32_t stage_bytes;  // one stage: the weight tile (kGemvJobRows x 256 bytes), then b_rows token rows
  int32_t s_bytes;      // one job's scale area
  int32_t zero_acc;     // up phase: zero acc before use
  int32_t pre_rows;     // rows of one split's pre-activation slice (>= pairs whenever K is split)
  int32_t pre_slices;   // split slices in pre (the up phase splits K at most this many ways; 0 = kMaxKSplit)
  int32_t* job_next;    // [2] job counters of the up and down launches, zeroed by the kernel that wrote
                        // the items (dispatch, table items, shared gate)
  int64_t tma_base;     // warp-streamed GEMV: base of its weight tensor maps (moeb200_expert_table.tma_base)
};

// Geometry shared by host and device.
constexpr int kGemvCons = 8;                  // consumer warps of a GEMV CTA
constexpr int kGemvJobRows = 32 * kGemvCons;  // weight rows of one job (up: 128 gate + 128 up)
constexpr int kGemvThreads = 32 * (kGemvCons + 1);
constexpr int kGemvStages = 2;
constexpr int kStepBytes = 256;  // bytes of one weight row per pipeline stage (multiple of 128)
constexpr int kSplitCols = 512;  // K splits are multiples of this many columns
constexpr int kMaxKSplit = 8;    // K splits of one GEMV launch at most

// weight tile of a stage: kStepBytes / 128 box columns, each 128 bytes of all kGemvJobRows rows
constexpr int kGemvWBytes = kGemvJobRows * kStepBytes;
constexpr int kGemvBoxCol = kGemvJobRows * 128;  // bytes between two box columns of a tile
static_assert(kStepBytes % 128 == 0 && kGemvBoxCol == (1 << 15), "box columns are 32 KB apart");
constexpr int kGemvMaxGrid = 160;                        // tensor-map slots are carved for this many CTAs
constexpr int kTmapSlots = 16;  // 128-byte tensor-map slots per CTA in the tensor-map workspace

__host__ __device__ inline int gemv_wbits(int wtype) {
  return wtype == MOEB200_I4 ? 4 : wtype == MOEB200_I8 ? 8 : wtype == MOEB200_F32 ? 32 : 16;
}

// Bytes of one token row in a stage (the stage's columns in a 16-bit activation type, padded to an
// odd multiple of 16 bytes so the token rows a warp reads at once fall in different banks).
__host__ __device__ inline int gemv_b_stride(int wtype) {
  return kStepBytes * 8 / gemv_wbits(wtype) * 2 + 16;
}

// Fused decode kernel (decode.cu): gate/up + SwiGLU + down + combine + cast in one launch, for work
// items of at most 8 pairs numbered slot-major. Counters (zeroed by the kernel that writes the
// items): ctr[1] CTAs that cleared acc, ctr[2] CTAs done; updone[max_items] gate/up units finished
// per item. slot_items[P + 1]: first item of each precision slot, then the item count.
struct DecodeParams {
  const Item* items;
  const int32_t* n_items;
  const int32_t* pos;      // sorted pair list: flat positions t*k + j
  const float* wflat;      // [T*k] router weights
  int32_t k;
  int32_t H;
  int32_t I;
  int32_t T;               // rows of acc (and out)
  const void* x;           // [tokens, H] activations
  void* h;                 // [n_pairs, I] activations, row j = sorted pair j
  float* acc;              // [T, H] fp32 combine buffer (the result itself when out is null)
  void* out;               // [T, H] activation type, or null
  int32_t add;             // out += instead of out =
  int32_t max_items;
  int32_t* status;
  int32_t* ctr;
  int32_t* updone;
  const int32_t* slot_items;
  int32_t nprec;
  int64_t tma_base;        // base of the weight tensor maps (moeb200_expert_table.tma_base)
  LayoutDev lay[4];
};
// Words of the decode kernel's counter region, zeroed with the items: ctr[4], slot_items[5] (padded
// to 12), then updone[max_items].
constexpr int kDecSlotItems = 4;
constexpr int kDecUpdone = 16;
inline int64_t decode_cnt_ints(int64_t max_items, int H) {
  (void)H;
  return kDecUpdone + max_items;
}
bool decode_supported(const moeb200_layout* lays, int nlay, int act_type, int H, int I);
cudaError_t launch_decode(const DecodeParams& p, const moeb200_layout* lays, int nlay, int act_type, int grid,
                          cudaStream_t s);

// Warp-streamed grouped GEMV (gemv_ws.cu): items of at most 8 pairs; int4 / int8 records with
// 64-column groups, or float records of the activation type; H and I multiples of 512; records on
// 4096-byte multiples above GemvParams::tma_base (row pitches dividing 4096 and the field offsets).
bool ws_supported(const moeb200_layout* lays, int nlay, int act_type, int H, int I, int max_item_pairs);
cudaError_t launch_ws_phases(GemvParams& p, const moeb200_layout* lays, int nlay, int act_type, int max_items,
                             cudaStream_t s);

// host launchers (gemv.cu)
// Plans split-K and the shared-memory geometry of the two GEMV phases, then launches gate/up and
// down (with trace marks around them). nb: token blocks of 8 per item (1 or 2).
cudaError_t launch_gemv_phases(GemvParams& p, const moeb200_layout* lays, int nlay, int act_type, int nb,
                               int max_items, int n_pairs, int max_split_pairs, cudaStream_t s);
cudaError_t launch_finalize(const float* acc, void* out, int act_type, int64_t n, int add, cudaStream_t s);
cudaError_t launch_combine_parts(const float* parts, int G, int64_t n, int act_type, void* out, int add,
                                 cudaStream_t s);
// trace hook of capi.cu: records a phase mark on the stream when tracing is on
cudaError_t trace_mark(int which, cudaStream_t s);
int num_sms_cached();
// tcgen05 grouped GEMM (gemm_tc.cu): items of up to 128 pairs, I and H multiples of 128
// (n_pairs: rows of h, the B operand of the down phase)
cudaError_t launch_gemm_up(const GemvParams& p, const moeb200_layout* lays, int nlay, int act_type, int n_pairs,
                           int grid, cudaStream_t s);
cudaError_t launch_gemm_down(const GemvParams& p, const moeb200_layout* lays, int nlay, int act_type, int n_pairs,
                             int grid, cudaStream_t s);

}  // namespace moeb200
