// Router / levels / dispatch declarations.
#pragma once

#include "gemv.cuh"

namespace moeb200 {

constexpr int kDispBlock = 1024;  // pairs per dispatch block
constexpr int kMaxKeys = 4096;    // max E * P (and E) handled by one dispatch
constexpr int kDispLoadThreads = 256;  // threads of a dispatch-count block (one warp ranks)

struct PolicyDev {
  int32_t mode;  // 0 hi, 1 lo, 2 hobbit, 3 threshold
  float t1;
  float t_mid;   // < 0: unset
  float t2;      // < 0: unset
  float thr;
};

struct LayoutOffs {
  int64_t gu_q, gu_s, dn_q, dn_s;
};

struct DispatchParams {
  const int64_t* idx;     // [T*k]
  const uint8_t* level;   // [T*k] or null
  const uint8_t* skip;    // [T*k] or null
  int32_t T, k, E, P;
  int32_t e_lo, e_hi;     // experts kept by this dispatch (expert parallelism); others are dropped
  int32_t nblk;           // ceil(T*k / kDispBlock)
  int32_t nt;             // max pairs per work item
  // outputs
  int32_t* counts_e;      // [E]
  int32_t* pos_e;         // [T*k]
  int32_t* counts_k;      // [E*P]
  int32_t* offs_k;        // [E*P] first sorted position of each key
  int32_t* offs_e;        // [E]   first sorted position of each expert (scratch)
  int32_t* pos_k;         // [T*k]
  int32_t* n_kept;        // [1] or null
  // scratch
  int32_t* blk_k;         // [nblk, E*P]
  int32_t* blk_e;         // [nblk, E]
  int32_t* rank_k;        // [T*k]
  int32_t* rank_e;        // [T*k]
  // work items (null: plain dispatch)
  Item* items;            // [T*k]
  int32_t* n_items;       // [1]
  const int64_t* table;   // [P, E] record addresses (0 = not resident) or null
  LayoutOffs offs[4];
  int32_t* miss;          // [1] pairs routed to a non-resident record, or null
  int32_t* status;
  int32_t* job_next;      // [2] GEMV job counters to zero with the items, or null
  int32_t* zero_cnt;      // [zero_n] split-K arrival counters to zero with the items, or null
  int32_t zero_n;
  int32_t* slot_items;    // [P + 1] first item of each precision slot (items are numbered slot-major)
                          // and the item count, or null
};

// shared_level >= 0: wr has E + 1 rows (the last one a shared expert's gate) and every token gets a
// (k + 1)-th pair (expert E, sigmoid of the gate logit, that level); outputs are [T, k + 1].
cudaError_t launch_router(const void* h, const void* wr, const float* bias, int act_type, int T, int H, int E, int k,
                          int renorm, float* logits, float* probs, float* w, int64_t* idx, const PolicyDev* pol,
                          uint8_t* level, uint8_t* skip, cudaStream_t s, int shared_level = -1);
cudaError_t launch_levels(const float* w, int T, int k, const PolicyDev& pol, uint8_t* level, uint8_t* skip,
                          cudaStream_t s);
cudaError_t launch_levels_vote(const int64_t* idx, uint8_t* level, const uint8_t* skip, int n, int E, double hi_vote,
                               cudaStream_t s);
cudaError_t launch_dispatch(const DispatchParams& p, cudaStream_t s);

}  // namespace moeb200
