// Router, precision levels and dispatch for the MoE layer on B200.
//
//  router_logits : logits[t, e] = round_to_model_dtype(sum_c h[t, c] * Wr[e, c]) (fp32 FMA chain per
//                  lane, fixed xor-tree across the warp), one warp per expert, tokens streamed.
//  router_topk   : one warp per token: + bias, fp32 softmax over all E, top-k by repeated warp
//                  arg-max (ties -> lower expert index), optional renormalisation, and the
//                  HOBBIT / threshold level of every pair (moelab/policy.py:77-137).
//  dispatch      : stable counting sort of the kept pairs by expert and by (expert, precision
//                  slot): per-block warp-aggregated histograms and in-order ranks (__match_any_sync),
//                  one scan over (key, block), then a scatter. Reproduces the reference's stable
//                  argsort + unique_consecutive (moelab/runtime.py:471-482) bit for bit, and emits the
//                  grouped-GEMV work items (<= 8*NB pairs of one (expert, slot) each).
#include "route.cuh"

namespace moeb200 {

namespace {

template <typename AT>
__device__ __forceinline__ float round_act(float v) {
  return to_f32<AT>(from_f32<AT>(v));
}

// ---- router logits --------------------------------------------------------------------------------
// One warp per tile of RE experts x RT tokens (a block of 8 warps = EG expert tiles x 8/EG token
// tiles, so its warps share the router rows and token rows in L1). For every (token, expert) lane l
// accumulates the columns l*8 + 256*i + j in that order in its own fp32 FMA chain; an xor butterfly
// over offsets 16..1 adds the 32 lane sums. The arithmetic of each logit is therefore the same for
// every tile shape (bit-exact with the single-token form).
// element j (0..7) of 8 packed 16-bit values, as fp32
template <typename AT>
__device__ __forceinline__ float elem8(const uint4& v, int j);
template <>
__device__ __forceinline__ float elem8<__nv_bfloat16>(const uint4& v, int j) {
  const uint32_t w = j < 2 ? v.x : j < 4 ? v.y : j < 6 ? v.z : v.w;
  return __uint_as_float((j & 1) ? (w & 0xffff0000u) : (w << 16));
}
template <>
__device__ __forceinline__ float elem8<__half>(const uint4& v, int j) {
  const uint32_t w = j < 2 ? v.x : j < 4 ? v.y : j < 6 ? v.z : v.w;
  return __half2float(__ushort_as_half((unsigned short)((j & 1) ? (w >> 16) : (w & 0xffffu))));
}

template <typename AT, int RE, int RT, int EG>
__global__ void __launch_bounds__(256) router_logits_kernel(const AT* __restrict__ h, const AT* __restrict__ wr,
                                                            int T, int H, int E, float* __restrict__ logits) {
  chain_wait();
  chain_release();
  constexpr int TG = 8 / EG;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e0 = (blockIdx.x * EG + warp % EG) * RE;
  const int t0 = (blockIdx.y * TG + warp / EG) * RT;
  if (e0 >= E || t0 >= T) return;
  const int ne = min(RE, E - e0), nt = min(RT, T - t0);
  float acc[RE][RT];
#pragma unroll
  for (int r = 0; r < RE; ++r)
#pragma unroll
    for (int q = 0; q < RT; ++q) acc[r][q] = 0.f;
  // raw 16-byte words of the step, converted element by element (a tile of RE x RT keeps RE + RT
  // words, not RE * 8 converted floats, in registers)
  // small tiles: eight column steps' loads in flight at once (a 2,048-column row in one L2 round trip)
  constexpr int kUnroll = RE * RT <= 4 ? 8 : 2;
#pragma unroll kUnroll
  for (int c = lane * 8; c < H; c += 256) {
    uint4 wv[RE], xv[RT];
#pragma unroll
    for (int r = 0; r < RE; ++r)
      wv[r] = r < ne ? __ldg(reinterpret_cast<const uint4*>(wr + (int64_t)(e0 + r) * H + c)) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int q = 0; q < RT; ++q)
      xv[q] = q < nt ? __ldg(reinterpret_cast<const uint4*>(h + (int64_t)(t0 + q) * H + c)) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float wf[RE], xf[RT];
#pragma unroll
      for (int r = 0; r < RE; ++r) wf[r] = elem8<AT>(wv[r], j);
#pragma unroll
      for (int q = 0; q < RT; ++q) xf[q] = elem8<AT>(xv[q], j);
#pragma unroll
      for (int r = 0; r < RE; ++r)
#pragma unroll
        for (int q = 0; q < RT; ++q) acc[r][q] = fmaf(xf[q], wf[r], acc[r][q]);
    }
  }
#pragma unroll
  for (int r = 0; r < RE; ++r)
#pragma unroll
    for (int q = 0; q < RT; ++q) {
      float a = acc[r][q];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      if (lane == 0 && r < ne && q < nt) logits[(int64_t)(t0 + q) * E + e0 + r] = round_act<AT>(a);
    }
}

// fp32 activations: 4 values per 16-byte load
__global__ void __launch_bounds__(256) router_logits_f32_kernel(const float* __restrict__ h,
                                                                const float* __restrict__ wr, int T, int H, int E,
                                                                int tok_per_block, float* __restrict__ logits) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x * 8 + warp;
  if (e >= E) return;
  const int t0 = blockIdx.y * tok_per_block;
  const int t1 = min(T, t0 + tok_per_block);
  const float* wrow = wr + (int64_t)e * H;
  for (int t = t0; t < t1; ++t) {
    const float* xrow = h + (int64_t)t * H;
    float acc = 0.f;
    for (int c = lane * 4; c < H; c += 128) {
      float4 wv = *reinterpret_cast<const float4*>(wrow + c);
      float4 xv = *reinterpret_cast<const float4*>(xrow + c);
      acc = fmaf(xv.x, wv.x, acc);
      acc = fmaf(xv.y, wv.y, acc);
      acc = fmaf(xv.z, wv.z, acc);
      acc = fmaf(xv.w, wv.w, acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) logits[(int64_t)t * E + e] = acc;
  }
}

// ---- precision levels of one token (one thread, k <= 32) ------------------------------------------
// Same operation order as the oracle restatement of PrecisionPolicy.unimportance/levels: the k
// weights are summed in index order, divided, ranked by descending weight (stable), and s is the
// running sum in rank order; the comparisons carry the reference's +1e-6 slack.
__device__ void token_levels(const float* w, int k, const PolicyDev& pol, uint8_t* level, uint8_t* skip) {
  if (pol.mode == 0 || pol.mode == 1) {
    for (int j = 0; j < k; ++j) {
      level[j] = pol.mode == 0 ? 0 : 2;
      if (skip) skip[j] = 0;
    }
    return;
  }
  if (pol.mode == 3) {
    for (int j = 0; j < k; ++j) {
      level[j] = w[j] >= pol.thr ? 0 : 2;
      if (skip) skip[j] = 0;
    }
    return;
  }
  float wn[32];
  float tot = 0.f;
  for (int j = 0; j < k; ++j) tot = __fadd_rn(tot, w[j]);
  tot = fmaxf(tot, 1e-12f);
  for (int j = 0; j < k; ++j) wn[j] = __fdiv_rn(w[j], tot);
  uint32_t used = 0;
  float acc = 0.f;
  const float t1 = pol.t1 + 1e-6f;
  const float tm = pol.t_mid + 1e-6f;
  const float t2 = pol.t2 + 1e-6f;
  for (int r = 0; r < k; ++r) {
    int best = -1;
    for (int j = 0; j < k; ++j)
      if (!(used >> j & 1u) && (best < 0 || wn[j] > wn[best])) best = j;
    used |= 1u << best;
    const float s = acc;
    acc = __fadd_rn(acc, wn[best]);
    uint8_t lv = 2;
    if (pol.t_mid >= 0.f && s <= tm) lv = 1;
    if (s <= t1) lv = 0;
    level[best] = lv;
    if (skip) skip[best] = (pol.t2 >= 0.f && s > t2 && lv != 0) ? 1 : 0;
  }
}

__global__ void levels_kernel(const float* __restrict__ w, int T, int k, PolicyDev pol, uint8_t* __restrict__ level,
                              uint8_t* __restrict__ skip) {
  chain_wait();
  chain_release();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  token_levels(w + (int64_t)t * k, k, pol, level + (int64_t)t * k, skip ? skip + (int64_t)t * k : nullptr);
}

// ---- per-expert precision vote (moelab/policy.py:148-154, applied per expert by
// moelab/runtime.py:476-488): over the kept pairs of expert e (n of them), the expert's level is the
// most precise L in (0, 1) with #(levels <= L) >= (hi_vote - 1e-9) * n (double arithmetic, as the
// reference's Python), else 2; every kept pair of e then takes that level. One CTA: the three
// counters of every expert live in shared memory. Pairs with an expert index outside [0, E) keep
// their level (the dispatch drops them and sets the status word).
__global__ void __launch_bounds__(1024) levels_vote_kernel(const int64_t* __restrict__ idx, uint8_t* __restrict__ level,
                                                           const uint8_t* __restrict__ skip, int n, int E,
                                                           double hi_vote) {
  extern __shared__ int32_t vc[];  // [E] kept pairs (then the vote), [E] levels <= 0, [E] levels <= 1
  chain_wait();
  chain_release();
  for (int i = threadIdx.x; i < 3 * E; i += blockDim.x) vc[i] = 0;
  __syncthreads();
  for (int p = threadIdx.x; p < n; p += blockDim.x) {
    if (skip && skip[p]) continue;
    const int64_t e = idx[p];
    if (e < 0 || e >= E) continue;
    const int l = level[p];
    atomicAdd(&vc[e], 1);
    if (l <= 0) atomicAdd(&vc[E + e], 1);
    if (l <= 1) atomicAdd(&vc[2 * E + e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const double need = (hi_vote - 1e-9) * (double)vc[e];
    vc[e] = (double)vc[E + e] >= need ? 0 : (double)vc[2 * E + e] >= need ? 1 : 2;
  }
  __syncthreads();
  for (int p = threadIdx.x; p < n; p += blockDim.x) {
    if (skip && skip[p]) continue;
    const int64_t e = idx[p];
    if (e < 0 || e >= E) continue;
    level[p] = (uint8_t)vc[e];
  }
}

// ---- softmax + top-k: one warp per token ------------------------------------------------------------
constexpr int kMaxEPerLane = 32;  // E <= 1024

// shared_level >= 0: logits rows hold E + 1 columns, the last one the shared expert's gate logit;
// every token gets one more pair after its k routed ones: (expert E, sigmoid(gate logit), level
// shared_level, not skipped), so outputs are [T, k + 1].
__global__ void __launch_bounds__(256) router_topk_kernel(const float* __restrict__ logits,
                                                          const float* __restrict__ bias, int T, int E, int k,
                                                          int renorm, float* __restrict__ probs,
                                                          float* __restrict__ w, int64_t* __restrict__ idx,
                                                          PolicyDev pol, int with_levels,
                                                          uint8_t* __restrict__ level, uint8_t* __restrict__ skip,
                                                          int shared_level) {
  chain_wait();
  chain_release();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= T) return;
  const int per = (E + 31) / 32;
  const int ls = shared_level >= 0 ? E + 1 : E;  // logits row stride
  const int kk = shared_level >= 0 ? k + 1 : k;  // output row stride
  float v[kMaxEPerLane];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < kMaxEPerLane; ++i) {
    if (i >= per) break;
    const int e = lane + 32 * i;
    float l = -INFINITY;
    if (e < E) {
      l = logits[(int64_t)t * ls + e];
      if (bias) l = __fadd_rn(l, bias[e]);
    }
    v[i] = l;
    m = fmaxf(m, l);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float ex[kMaxEPerLane];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxEPerLane; ++i) {
    if (i >= per) break;
    const int e = lane + 32 * i;
    ex[i] = e < E ? expf(v[i] - m) : 0.f;
    s += ex[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  // top-k on the logits (softmax is strictly increasing in the logit): arg-max rounds with the
  // lower index winning ties.
  uint32_t taken = 0;
  float wsel = 0.f;  // lane j < k holds the j-th selected probability
  int isel = 0;
  for (int r = 0; r < k; ++r) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kMaxEPerLane; ++i) {
      if (i >= per) break;
      const int e = lane + 32 * i;
      if (e < E && !(taken >> i & 1u) && (v[i] > bv || (v[i] == bv && e < bi))) {
        bv = v[i];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    const int owner = bi & 31;
    // fetch the owner's exp value for expert bi
    float mine = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxEPerLane; ++i) {
      if (i >= per) break;
      if (lane + 32 * i == bi) mine = ex[i];
    }
    const float ebi = __shfl_sync(0xffffffffu, mine, owner);
    if (lane == r) {
      wsel = __fdiv_rn(ebi, s);
      isel = bi;
    }
  }
  if (probs) {
#pragma unroll
    for (int i = 0; i < kMaxEPerLane; ++i) {
      if (i >= per) break;
      const int e = lane + 32 * i;
      if (e < E) probs[(int64_t)t * E + e] = __fdiv_rn(ex[i], s);
    }
  }
  if (renorm) {
    float tot = 0.f;
    for (int j = 0; j < k; ++j) tot = __fadd_rn(tot, __shfl_sync(0xffffffffu, wsel, j));
    wsel = __fdiv_rn(wsel, tot);
  }
  if (lane < k) {
    w[(int64_t)t * kk + lane] = wsel;
    idx[(int64_t)t * kk + lane] = isel;
  }
  if (shared_level >= 0 && lane == 0) {
    // the gate logit is already rounded to the activation dtype (as F.linear returns it)
    const float gl = logits[(int64_t)t * ls + E];
    w[(int64_t)t * kk + k] = 1.0f / (1.0f + expf(-gl));
    idx[(int64_t)t * kk + k] = E;
  }
  if (with_levels) {
    if (pol.mode != 2) {
      // hi / lo / threshold: a pair's level depends on its own weight only, which lane j holds
      if (lane < k) {
        level[(int64_t)t * kk + lane] = pol.mode == 0 ? 0 : pol.mode == 1 ? 2 : (wsel >= pol.thr ? 0 : 2);
        if (skip) skip[(int64_t)t * kk + lane] = 0;
      }
    } else {
      // HOBBIT ranks the token's pairs: lane 0 gathers the k weights from their lanes (no read-back
      // from global memory) and runs the serial rule
      float wl[32];
      for (int j = 0; j < k; ++j) {
        const float v = __shfl_sync(0xffffffffu, wsel, j);
        if (lane == 0) wl[j] = v;
      }
      if (lane == 0) token_levels(wl, k, pol, level + (int64_t)t * kk, skip ? skip + (int64_t)t * kk : nullptr);
    }
    if (shared_level >= 0 && lane == 0) {
      level[(int64_t)t * kk + k] = (uint8_t)shared_level;
      if (skip) skip[(int64_t)t * kk + k] = 0;
    }
  }
}

// ---- dispatch ----------------------------------------------------------------------------------------
__device__ __forceinline__ int slot_of(int level, int P) {
  if (P >= 3) return min(level, P - 1);
  return level == 0 ? 0 : P - 1;
}

// One warp ranks the n pairs of a dispatch block in order, 32 at a time: each pair's rank among the
// earlier pairs with the same key (expert*P + slot, and expert); cnt_k/cnt_e count the pairs so far.
__device__ __forceinline__ void rank_in_order(int lane, int n, const int32_t* key_s, const int32_t* e_s,
                                              int32_t* cnt_k, int32_t* cnt_e, int32_t* rank_k, int32_t* rank_e) {
  for (int c = 0; c < n; c += 32) {
    const int i = c + lane;
    int key = -1, e = -1;
    if (i < n) {
      key = key_s[i];
      e = e_s[i];
    }
    const uint32_t lt = (1u << lane) - 1u;
    const uint32_t mk = __match_any_sync(0xffffffffu, key);
    const uint32_t me = __match_any_sync(0xffffffffu, e);
    int rk = 0, re = 0;
    if (key >= 0) {
      rk = cnt_k[key] + __popc(mk & lt);
      re = cnt_e[e] + __popc(me & lt);
    }
    __syncwarp();
    // the highest lane of each group publishes the new count
    if (key >= 0 && (mk >> lane) == 1u) cnt_k[key] = rk + 1;
    if (e >= 0 && (me >> lane) == 1u) cnt_e[e] = re + 1;
    __syncwarp();
    if (i < n) {
      rank_k[i] = key >= 0 ? rk : -1;
      rank_e[i] = re;
    }
  }
}

// Key (expert*P + slot) and expert of pair i, or -1 for a dropped pair (skipped, or routed to an
// expert outside [e_lo, e_hi)); an index outside [0, E) sets the status word.
__device__ __forceinline__ void pair_key(const DispatchParams& p, int i, int& key, int& e) {
  key = -1;
  e = -1;
  const bool skipped = p.skip && p.skip[i];
  const int64_t ev = p.idx[i];
  if (ev < 0 || ev >= p.E) {
    if (p.status) atomicExch(p.status, kDevBadIndex);
  } else if (!skipped && ev >= p.e_lo && ev < p.e_hi) {
    e = (int)ev;
    const int lv = p.level ? p.level[i] : 0;
    key = e * p.P + slot_of(lv, p.P);
  }
}

// D1: one warp per block of kDispBlock pairs, processed in order 32 at a time. Each pair gets its
// rank among the earlier pairs of the block with the same key (expert, and expert*P + slot).
__global__ void __launch_bounds__(kDispLoadThreads) dispatch_count_kernel(DispatchParams p) {
  chain_wait();
  chain_release();
  extern __shared__ int32_t sh[];
  int32_t* cnt_k = sh;               // [E*P]
  int32_t* cnt_e = sh + p.E * p.P;   // [E]
  const int tid = threadIdx.x, lane = tid & 31;
  const int keys = p.E * p.P;
  for (int i = tid; i < keys + p.E; i += blockDim.x) sh[i] = 0;
  const int n = p.T * p.k;
  const int b = blockIdx.x;
  const int base = b * kDispBlock;
  const int end = min(n, base + kDispBlock);
  // keys of the whole block first, loaded by all threads; one warp ranks them in order below
  int32_t* key_s = sh + keys + p.E;   // [kDispBlock]
  int32_t* e_s = key_s + kDispBlock;  // [kDispBlock]
  for (int i = base + tid; i < end; i += blockDim.x) {
    int key, e;
    pair_key(p, i, key, e);
    key_s[i - base] = key;
    e_s[i - base] = e;
  }
  __syncthreads();
  if (tid >= 32) return;
  rank_in_order(lane, end - base, key_s, e_s, cnt_k, cnt_e, p.rank_k + base, p.rank_e + base);
  __syncwarp();
  for (int i = lane; i < keys; i += 32) p.blk_k[(int64_t)b * keys + i] = cnt_k[i];
  for (int i = lane; i < p.E; i += 32) p.blk_e[(int64_t)b * p.E + i] = cnt_e[i];
}

// Block-wide exclusive scan of up to 1024 * kScanPer values (one block of 1024 threads).
template <int PER>
__device__ int32_t block_exclusive_scan(int32_t (&v)[PER], int32_t* sh_warp) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int32_t loc = 0;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int32_t x = v[i];
    v[i] = loc;
    loc += x;
  }
  int32_t inc = loc;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  if (lane == 31) sh_warp[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    int32_t s = lane < (int)(blockDim.x >> 5) ? sh_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    sh_warp[lane] = s;
  }
  __syncthreads();
  const int32_t before = (warp > 0 ? sh_warp[warp - 1] : 0) + inc - loc;
#pragma unroll
  for (int i = 0; i < PER; ++i) v[i] += before;
  const int32_t total = sh_warp[31];
  __syncthreads();
  return total;
}

// Per-key totals, first positions (exclusive scans) and work items, by one block of 1024 threads.
// With cnt_k/cnt_e (a single dispatch block whose counts are in shared memory) the totals are read
// there and the first positions are also left in offk_s/offe_s; otherwise the per-block counts in
// global memory are turned into per-(block, key) prefixes on the way.
constexpr int kKeysPerThread = kMaxKeys / 1024;  // slot-major keys of each thread of a 1024-thread block

// Record address of each of the thread's slot-major keys m = slot * E + expert (the table's own
// index; 0 = not resident or no table), loaded first so that the load overlaps the pair loads
__device__ __forceinline__ void load_key_records(const DispatchParams& p, int64_t (&rec)[kKeysPerThread]) {
  const int keys = p.E * p.P;
#pragma unroll
  for (int i = 0; i < kKeysPerThread; ++i) {
    const int m = threadIdx.x * kKeysPerThread + i;
    rec[i] = (p.items != nullptr && p.table != nullptr && m < keys) ? p.table[m] : 0;
  }
}

// rec_pre: the thread's key records from load_key_records
__device__ void finish_keys(const DispatchParams& p, const int32_t* cnt_k, const int32_t* cnt_e, int32_t* offk_s,
                            int32_t* offe_s, int32_t* sh_warp, const int64_t (&rec_pre)[kKeysPerThread]) {
  __shared__ int32_t tot_s[kMaxKeys];    // pairs per key
  __shared__ int32_t offk_sh[kMaxKeys];  // first sorted position per key
  const int keys = p.E * p.P;
  const int tid = threadIdx.x;
  if (tid == 0 && p.miss) *p.miss = 0;
  for (int i = tid; i < p.zero_n; i += blockDim.x) p.zero_cnt[i] = 0;
  __syncthreads();
  constexpr int PER = kKeysPerThread;
  int32_t tot_k[PER], tot_e[PER], nit[PER];
  int64_t rec_i[PER];  // record address of each of the thread's slot-major keys (loaded once)
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int key = tid * PER + i;
    int32_t run = 0;
    if (key < keys) {
      if (cnt_k) {
        run = cnt_k[key];
      } else {
        for (int b0 = 0; b0 < p.nblk; b0 += 8) {  // 8 independent loads in flight
          int32_t cv[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) cv[u] = b0 + u < p.nblk ? p.blk_k[(int64_t)(b0 + u) * keys + key] : 0;
#pragma unroll
          for (int u = 0; u < 8; ++u)
            if (b0 + u < p.nblk) {
              p.blk_k[(int64_t)(b0 + u) * keys + key] = run;
              run += cv[u];
            }
        }
      }
    }
    tot_k[i] = key < keys ? run : 0;
    int32_t rune = 0;
    const int e = tid * PER + i;
    if (e < p.E) {
      if (cnt_e) {
        rune = cnt_e[e];
      } else {
        for (int b0 = 0; b0 < p.nblk; b0 += 8) {
          int32_t cv[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) cv[u] = b0 + u < p.nblk ? p.blk_e[(int64_t)(b0 + u) * p.E + e] : 0;
#pragma unroll
          for (int u = 0; u < 8; ++u)
            if (b0 + u < p.nblk) {
              p.blk_e[(int64_t)(b0 + u) * p.E + e] = rune;
              rune += cv[u];
            }
        }
      }
    }
    tot_e[i] = e < p.E ? rune : 0;
    if (key < keys) tot_s[key] = run;
  }
  __syncthreads();
  // work items, numbered slot-major (every slot-0 record's items first: the largest records, so a
  // round-robin of jobs over the CTAs hands the heavy ones out first); only resident records
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int m = tid * PER + i;  // slot-major index sl * E + ex
    int32_t ni = 0;
    int64_t rec = 0;
    if (p.items != nullptr && m < keys) {
      const int sl = m / p.E, ex = m % p.E;
      const int32_t run = tot_s[ex * p.P + sl];
      if (run > 0) {
        rec = p.table ? rec_pre[i] : 0;  // p.table[sl * E + ex]
        if (rec != 0 || !p.table) ni = (run + p.nt - 1) / p.nt;
        else if (p.miss) atomicAdd(p.miss, run);
      }
    }
    nit[i] = ni;
    rec_i[i] = rec;
  }
  int32_t off_k[PER], off_e[PER], off_i[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    off_k[i] = tot_k[i];
    off_e[i] = tot_e[i];
    off_i[i] = nit[i];
  }
  const int32_t n_kept = block_exclusive_scan<PER>(off_k, sh_warp);
  block_exclusive_scan<PER>(off_e, sh_warp);
  const int32_t n_items = block_exclusive_scan<PER>(off_i, sh_warp);
  if (p.slot_items) {  // slot s's items start at key s*E (slot-major numbering)
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int m = tid * PER + i;
      if (m < keys && m % p.E == 0) p.slot_items[m / p.E] = off_i[i];
    }
    if (tid == 0) p.slot_items[p.P] = n_items;
  }
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int key = tid * PER + i;
    if (key < keys) {
      p.counts_k[key] = tot_k[i];
      p.offs_k[key] = off_k[i];
      offk_sh[key] = off_k[i];
      if (offk_s) offk_s[key] = off_k[i];
    }
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int m = tid * PER + i;
    if (nit[i] > 0) {
      const int sl = m / p.E, ex = m % p.E;
      const int key = ex * p.P + sl;
      const int64_t rec = rec_i[i];
      const LayoutOffs lo = p.offs[sl];
      const int32_t run = tot_s[key];
      for (int q = 0; q < nit[i]; ++q) {
        Item it;
        it.p_guq = rec + lo.gu_q;
        it.p_gus = rec + lo.gu_s;
        it.p_dnq = rec + lo.dn_q;
        it.p_dns = rec + lo.dn_s;
        it.slot = sl;
        it.start = offk_sh[key] + q * p.nt;
        it.ntok = min(p.nt, run - q * p.nt);
        it._pad = ex;
        p.items[off_i[i] + q] = it;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = tid * PER + i;
    if (e < p.E) {
      p.counts_e[e] = tot_e[i];
      p.offs_e[e] = off_e[i];
      if (offe_s) offe_s[e] = off_e[i];
    }
  }
  if (tid == 0) {
    if (p.n_items) *p.n_items = n_items;
    if (p.n_kept) *p.n_kept = n_kept;
    if (p.job_next) {
      p.job_next[0] = 0;
      p.job_next[1] = 0;
    }
  }
}

// D2: one block of 1024 threads over the per-block counts of D1.
__global__ void __launch_bounds__(1024) dispatch_scan_kernel(DispatchParams p) {
  __shared__ int32_t sh_warp[32];
  chain_wait();
  chain_release();
  int64_t rec[kKeysPerThread];
  load_key_records(p, rec);
  finish_keys(p, nullptr, nullptr, nullptr, nullptr, sh_warp, rec);
}

// D1+D2+D3 in one block of 1024 threads when all pairs fit one dispatch block (T*k <= kDispBlock):
// keys; per-key and per-expert totals by shared-memory atomics (any order); totals/positions/items;
// each pair dropped into its key's and its expert's bucket at the slot its atomic returned; then
// each pair's in-order rank is the number of smaller pair indices in its bucket (a bucket holds at
// most T pairs: a token routes to k distinct experts), which fixes the stable sorted order.
__global__ void __launch_bounds__(1024) dispatch_fused_kernel(DispatchParams p) {
  extern __shared__ int32_t sh[];
  __shared__ int32_t sh_warp[32];
  chain_wait();
  chain_release();
  int64_t rec[kKeysPerThread];
  load_key_records(p, rec);
  const int keys = p.E * p.P;
  int32_t* cnt_k = sh;                 // [keys]
  int32_t* cnt_e = cnt_k + keys;       // [E]
  int32_t* offk = cnt_e + p.E;         // [keys]
  int32_t* offe = offk + keys;         // [E]
  int32_t* bk_s = offe + p.E;          // [kDispBlock] pair indices bucketed by key (unordered in a bucket)
  int32_t* be_s = bk_s + kDispBlock;   // [kDispBlock] pair indices bucketed by expert
  const int tid = threadIdx.x;
  const int n = p.T * p.k;
  for (int i = tid; i < keys + p.E; i += blockDim.x) sh[i] = 0;
  int key = -1, e = -1;
  if (tid < n) pair_key(p, tid, key, e);
  __syncthreads();
  int sk = 0, se = 0;
  if (key >= 0) {
    sk = atomicAdd(&cnt_k[key], 1);
    se = atomicAdd(&cnt_e[e], 1);
  }
  __syncthreads();
  finish_keys(p, cnt_k, cnt_e, offk, offe, sh_warp, rec);
  __syncthreads();
  if (key >= 0) {
    bk_s[offk[key] + sk] = tid;
    be_s[offe[e] + se] = tid;
  }
  __syncthreads();
  if (key >= 0) {
    const int k0 = offk[key], kn = cnt_k[key];
    int rk = 0;
    for (int q = 0; q < kn; ++q) rk += bk_s[k0 + q] < tid;
    const int e0 = offe[e], en = cnt_e[e];
    int re = 0;
    for (int q = 0; q < en; ++q) re += be_s[e0 + q] < tid;
    p.pos_k[k0 + rk] = tid;
    p.pos_e[e0 + re] = tid;
  }
}

// D3: scatter each kept pair to its sorted positions.
__global__ void dispatch_scatter_kernel(DispatchParams p) {
  chain_wait();
  chain_release();
  const int n = p.T * p.k;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int rk = p.rank_k[i];
  if (rk < 0) return;
  const int b = i / kDispBlock;
  const int e = (int)p.idx[i];
  const int lv = p.level ? p.level[i] : 0;
  const int key = e * p.P + slot_of(lv, p.P);
  p.pos_k[p.offs_k[key] + p.blk_k[(int64_t)b * p.E * p.P + key] + rk] = i;
  p.pos_e[p.offs_e[e] + p.blk_e[(int64_t)b * p.E + e] + p.rank_e[i]] = i;
}

}  // namespace

cudaError_t launch_router(const void* h, const void* wr, const float* bias, int act_type, int T, int H, int E_route,
                          int k, int renorm, float* logits, float* probs, float* w, int64_t* idx, const PolicyDev* pol,
                          uint8_t* level, uint8_t* skip, cudaStream_t s, int shared_level) {
  const int E = shared_level >= 0 ? E_route + 1 : E_route;  // logit columns (router rows of wr)
  const int tpb = T <= 8 ? T : 8;
  dim3 grid((E + 7) / 8, (T + tpb - 1) / tpb);
  // few (token, expert) logits: one expert x 4 tokens per warp (8 experts per block) keeps every SM
  // busy; many: 4 x 8 per warp (8 x 32 per block) cuts the L2 re-reads of token and router rows
  // prefill-sized: 8 x 8 per warp (16 experts x 32 tokens per block) keeps 64 FMA chains per lane
  const bool huge = (int64_t)T * E >= 262144;
  const bool big = (int64_t)T * E >= 65536;
  const dim3 g16 = huge  ? dim3((E + 15) / 16, (T + 31) / 32)
                   : big ? dim3((E + 7) / 8, (T + 31) / 32)
                         : dim3((E + 7) / 8, (T + 3) / 4);
  cudaError_t e = cudaSuccess;
  if (act_type == MOEB200_F16) {
    const __half* ha = static_cast<const __half*>(h);
    const __half* wa = static_cast<const __half*>(wr);
    if (huge)
      e = launch_chained(router_logits_kernel<__half, 8, 8, 2>, g16, 256, 0, s, ha, wa, T, H, E, logits);
    else if (big)
      e = launch_chained(router_logits_kernel<__half, 4, 8, 2>, g16, 256, 0, s, ha, wa, T, H, E, logits);
    else
      e = launch_chained(router_logits_kernel<__half, 1, 4, 8>, g16, 256, 0, s, ha, wa, T, H, E, logits);
  } else if (act_type == MOEB200_BF16) {
    const __nv_bfloat16* ha = static_cast<const __nv_bfloat16*>(h);
    const __nv_bfloat16* wa = static_cast<const __nv_bfloat16*>(wr);
    if (huge)
      e = launch_chained(router_logits_kernel<__nv_bfloat16, 8, 8, 2>, g16, 256, 0, s, ha, wa, T, H, E, logits);
    else if (big)
      e = launch_chained(router_logits_kernel<__nv_bfloat16, 4, 8, 2>, g16, 256, 0, s, ha, wa, T, H, E, logits);
    else
      e = launch_chained(router_logits_kernel<__nv_bfloat16, 1, 4, 8>, g16, 256, 0, s, ha, wa, T, H, E, logits);
  } else {
    router_logits_f32_kernel<<<grid, 256, 0, s>>>(static_cast<const float*>(h), static_cast<const float*>(wr), T, H,
                                                  E, tpb, logits);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return e;
  PolicyDev pd{};
  if (pol) pd = *pol;
  return launch_chained(router_topk_kernel, dim3((T + 7) / 8), dim3(256), 0, s, logits, bias, T, E_route, k, renorm,
                        probs, w, idx, pd, (int)(pol != nullptr), level, skip, shared_level);
}

cudaError_t launch_levels(const float* w, int T, int k, const PolicyDev& pol, uint8_t* level, uint8_t* skip,
                          cudaStream_t s) {
  return launch_chained(levels_kernel, dim3((T + 127) / 128), dim3(128), 0, s, w, T, k, pol, level, skip);
}

cudaError_t launch_levels_vote(const int64_t* idx, uint8_t* level, const uint8_t* skip, int n, int E, double hi_vote,
                               cudaStream_t s) {
  const size_t sh = (size_t)3 * E * sizeof(int32_t);
  cudaError_t e = cudaFuncSetAttribute(levels_vote_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sh);
  if (e != cudaSuccess) return e;
  return launch_chained(levels_vote_kernel, dim3(1), dim3(1024), sh, s, idx, level, skip, n, E, hi_vote);
}

cudaError_t launch_dispatch(const DispatchParams& p, cudaStream_t s) {
  const int keys = p.E * p.P;
  if (p.nblk == 1) {
    const size_t shf = (size_t)(2 * (keys + p.E) + 2 * kDispBlock) * sizeof(int32_t);
    cudaError_t e = cudaFuncSetAttribute(dispatch_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)shf);
    if (e != cudaSuccess) return e;
    return launch_chained(dispatch_fused_kernel, dim3(1), dim3(1024), shf, s, p);
  }
  const size_t sh = (size_t)(keys + p.E + 2 * kDispBlock) * sizeof(int32_t);
  cudaError_t e = launch_chained(dispatch_count_kernel, dim3(p.nblk), dim3(kDispLoadThreads), sh, s, p);
  if (e != cudaSuccess) return e;
  e = launch_chained(dispatch_scan_kernel, dim3(1), dim3(1024), 0, s, p);
  if (e != cudaSuccess) return e;
  const int n = p.T * p.k;
  return launch_chained(dispatch_scatter_kernel, dim3((n + 255) / 256), dim3(256), 0, s, p);
}

}  // namespace moeb200
