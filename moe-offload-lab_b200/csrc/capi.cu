// extern "C" entry points of libmoeb200 (declared in include/moeb200.h).
//
// Host-side validation, workspace carving and kernel sequencing. Nothing here allocates device
// memory, synchronises a stream (except moeb200_check_workspace) or reads device data, so every
// entry point can be recorded in a CUDA graph.
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "route.cuh"

using namespace moeb200;

namespace {

thread_local std::string g_err;
thread_local int g_err_code = MOEB200_OK;
// Phase tracing (measurement): while on, every grouped-expert call records library-owned CUDA
// events before the gate/up phase, between the phases and after the down phase.
struct TraceRec {
  cudaEvent_t ev[3];
};
thread_local bool g_tracing = false;
thread_local std::vector<TraceRec> g_trace_pool;
thread_local size_t g_trace_used = 0;

// Average routed pairs per expert from which the automatic path takes the tcgen05 GEMM.
constexpr int64_t kGemmPairsPerExpert = 40;

// Expert-product path of the next calls on this thread: 0 auto, 1 grouped GEMV, 2 tcgen05 GEMM,
// 3 fused decode kernel, 4 warp-streamed grouped GEMV.
thread_local int g_path = 0;
thread_local int g_item_tokens = 0;  // GEMV work-item size: 0 = automatic, else 8 or 16
thread_local int g_last_path = 0;    // path of the thread's last experts_forward call (moeb200_path_used)

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  g_err_code = code;
  return code;
}

#define CUDA_TRY(expr)                                                                       \
  do {                                                                                       \
    cudaError_t e_ = (expr);                                                                 \
    if (e_ != cudaSuccess) return fail(MOEB200_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(e_)); \
  } while (0)

constexpr size_t kAlign = 256;

// Workspace carving: the same walk sizes (base == nullptr) and hands out sub-buffers.
struct Carve {
  uint8_t* base;
  size_t off = 0;
  explicit Carve(void* b) : base(static_cast<uint8_t*>(b)) {}
  template <typename T>
  T* take(size_t count) {
    off = (off + kAlign - 1) / kAlign * kAlign;
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += count * sizeof(T);
    return p;
  }
};

// Header of every workspace: status word and small device counters.
struct WsHeader {
  int32_t status;
  int32_t n_items;
  int32_t n_kept;
  int32_t miss;
  int32_t job_next[2];  // GEMV job counters (up, down), zeroed by the kernel that writes the items
  int32_t _pad[2];
};

int act_bytes(int act) { return act == MOEB200_F32 ? 4 : 2; }


bool is_int(int wt) { return wt == MOEB200_I4 || wt == MOEB200_I8; }

// Host mirror of the device chunk-kind choice (gemv.cu kind_of): returns false if unsupported.
bool matrix_supported(int wt, int K, int gs, const char* name, std::string& why) {
  char b[256];
  switch (wt) {
    case MOEB200_I4:
      if (gs > 0 && gs % 32 == 0 && K % 32 == 0 && K % gs == 0) return true;
      snprintf(b, sizeof b, "%s: int4 needs a group size multiple of 32 dividing K (K=%d, gs=%d)", name, K, gs);
      break;
    case MOEB200_I8:
      if (gs > 0 && gs % 16 == 0 && K % 16 == 0 && K % gs == 0) return true;
      snprintf(b, sizeof b, "%s: int8 needs a group size multiple of 16 dividing K (K=%d, gs=%d)", name, K, gs);
      break;
    case MOEB200_F16:
    case MOEB200_BF16:
    case MOEB200_F32:
      if (K % 16 == 0) return true;
      snprintf(b, sizeof b, "%s: float records need K %% 16 == 0 (K=%d)", name, K);
      break;
    default:
      snprintf(b, sizeof b, "%s: unknown record element type %d", name, wt);
  }
  why = b;
  return false;
}

int check_layout(const moeb200_layout& L, int H, int I) {
  if (L.hidden != H || L.inter != I)
    return fail(MOEB200_ERR_INVALID, "layouts disagree on shapes (%d,%d) vs (%d,%d)", L.hidden, L.inter, H, I);
  std::string why;
  if (!matrix_supported(L.wtype, H, L.gs_up, "gate_up", why)) return fail(MOEB200_ERR_UNSUPPORTED, "%s", why.c_str());
  if (!matrix_supported(L.wtype, I, L.gs_dn, "down", why)) return fail(MOEB200_ERR_UNSUPPORTED, "%s", why.c_str());
  if (L.off_gu_q < 0 || L.off_dn_q < 0 || (L.off_gu_q % 16) || (L.off_dn_q % 16))
    return fail(MOEB200_ERR_INVALID, "record field offsets must be 16-byte aligned");
  if (is_int(L.wtype) && (L.off_gu_s < 0 || L.off_dn_s < 0 || (L.off_gu_s % 16) || (L.off_dn_s % 16)))
    return fail(MOEB200_ERR_INVALID, "scale field offsets must be 16-byte aligned");
  return MOEB200_OK;
}

int check_shapes(int H, int I) {
  if (H <= 0 || I <= 0 || H % 32 != 0 || I % 16 != 0)
    return fail(MOEB200_ERR_UNSUPPORTED, "hidden must be a multiple of 32 and inter of 16 (H=%d, I=%d)", H, I);
  if (H % 8 || I % 8) return fail(MOEB200_ERR_UNSUPPORTED, "H and I must be multiples of 8");
  return MOEB200_OK;
}

// Split-K planning of the GEMV phases: a split covers a multiple of kSplitCols input columns (a
// multiple of every group size and pipeline step), and is only used for small pair counts (the
// pre-activation buffer holds kMaxKSplit slices of kMaxSplitPairs pairs). Splits only pay when the
// jobs would not fill the SMs, i.e. for a few hundred pairs at most.
constexpr int kMaxSplitPairs = 256;

// Split-K scratch of a call over n pairs: pre-activation rows per split slice, and arrival counters
// (zeroed by the kernel that writes the call's items).
int split_rows(int64_t n) { return (int)std::min<int64_t>(n, kMaxSplitPairs); }
size_t split_pre_floats(int64_t n, int I) { return (size_t)kMaxKSplit * split_rows(n) * 2 * I; }
int split_cnt_ints(int64_t n, int I) { return split_rows(n) * (I / 16); }

// Upper bound on the K splits the GEMV planner (gemv.cu plan_and_launch) can choose for n one-token
// items (the pointer-table entry points). The planner doubles the splits while the up jobs (n items x
// ceil(I / (kGemvJobRows/2)) row blocks) would not give every SM one, capped by the slices sized here;
// it may stop earlier (split_ok), never later, so the slices always suffice. Sizing them by this rule
// keeps small calls' scratch small. Keep the two rules in step.
int table_split_slices(int64_t n, int I) {
  constexpr int kUpRows = kGemvJobRows / 2;
  const int64_t jobs1 = std::max<int64_t>(1, n) * ((I + kUpRows - 1) / kUpRows);
  const int sms = num_sms_cached();
  int ks = 1;
  while (ks < kMaxKSplit && jobs1 * ks < sms) ks *= 2;
  return ks;
}


struct ForwardWs {
  WsHeader* hdr;
  int32_t *pos_e, *pos_k, *counts_e, *counts_k, *offs_k, *offs_e, *blk_k, *blk_e, *rank_k, *rank_e;
  Item* items;
  uint8_t* h;
  float* pre;
  int32_t* cnt;
  uint8_t* tmaps;
  float* acc;
  float* logits;
  size_t bytes;
};

ForwardWs carve_forward(void* base, int T, int k, int E, int P, int H, int I, int act) {
  Carve c(base);
  ForwardWs w{};
  const int n = T * k;
  const int keys = E * P;
  const int nblk = (n + kDispBlock - 1) / kDispBlock;
  w.hdr = c.take<WsHeader>(1);
  w.pos_e = c.take<int32_t>(n);
  w.pos_k = c.take<int32_t>(n);
  w.counts_e = c.take<int32_t>(E);
  w.counts_k = c.take<int32_t>(keys);
  w.offs_k = c.take<int32_t>(keys);
  w.offs_e = c.take<int32_t>(E);
  w.blk_k = c.take<int32_t>((size_t)nblk * keys);
  w.blk_e = c.take<int32_t>((size_t)nblk * E);
  w.rank_k = c.take<int32_t>(n);
  w.rank_e = c.take<int32_t>(n);
  w.items = c.take<Item>(n);
  w.h = c.take<uint8_t>((size_t)n * I * act_bytes(act));
  w.pre = c.take<float>(split_pre_floats(n, I));
  w.cnt = c.take<int32_t>((size_t)std::max<int64_t>(split_cnt_ints(n, I), decode_cnt_ints(n, H)));
  w.tmaps = c.take<uint8_t>((size_t)kTmapSlots * kGemvMaxGrid * 128);
  w.acc = c.take<float>((size_t)T * H);
  w.bytes = c.off;
  return w;
}

LayoutDev to_dev(const moeb200_layout& L) {
  LayoutDev d{};
  d.wtype = L.wtype;
  d.gs_up = L.gs_up;
  d.gs_dn = L.gs_dn;
  return d;
}

int run_expert_phases(GemvParams& gp, const moeb200_layout* lays, int nlay, int act, int max_items, int n_pairs,
                      int nt, cudaStream_t s, void* out, int add, bool gemm = false, bool streamed = false) {
  if (streamed) {
    CUDA_TRY(launch_ws_phases(gp, lays, nlay, act, max_items, s));
    if (out) CUDA_TRY(launch_finalize(gp.acc, out, act, (int64_t)gp.T * gp.H, add, s));
    return MOEB200_OK;
  }
  if (gemm) {
    const int sms = num_sms_cached();
    const int64_t tiles = (int64_t)max_items * (gp.I / 128);
    const int64_t tiles_dn = (int64_t)max_items * (gp.H / 128);
    const int grid_up = (int)std::max<int64_t>(1, std::min<int64_t>(sms, tiles));
    const int grid_dn = (int)std::max<int64_t>(1, std::min<int64_t>(sms, tiles_dn));
    CUDA_TRY(trace_mark(0, s));
    cudaError_t e = launch_gemm_up(gp, lays, nlay, act, n_pairs, grid_up, s);
    if (e == cudaErrorInvalidConfiguration)
      return fail(MOEB200_ERR_UNSUPPORTED, "GEMM: the record layouts need more shared memory than a CTA has");
    CUDA_TRY(e);
    CUDA_TRY(trace_mark(1, s));
    CUDA_TRY(launch_gemm_down(gp, lays, nlay, act, n_pairs, grid_dn, s));
    CUDA_TRY(trace_mark(2, s));
    if (out) CUDA_TRY(launch_finalize(gp.acc, out, act, (int64_t)gp.T * gp.H, add, s));
    return MOEB200_OK;
  }
  const int nb = nt > 8 ? 2 : 1;
  const cudaError_t e = launch_gemv_phases(gp, lays, nlay, act, nb, max_items, n_pairs, kMaxSplitPairs, s);
  if (e == cudaErrorInvalidConfiguration)
    return fail(MOEB200_ERR_UNSUPPORTED, "GEMV: the record layouts need more shared memory than a CTA has");
  CUDA_TRY(e);
  if (out) CUDA_TRY(launch_finalize(gp.acc, out, act, (int64_t)gp.T * gp.H, add, s));
  return MOEB200_OK;
}

__global__ void table_items_kernel(const int64_t* __restrict__ tab, const float* __restrict__ w, int n,
                                   Item* __restrict__ items, int32_t* __restrict__ n_items, int32_t* __restrict__ pos,
                                   int32_t* __restrict__ job_next, int32_t* __restrict__ cnt, int cnt_n) {
  for (int i = threadIdx.x; i < cnt_n; i += blockDim.x) cnt[i] = 0;  // split-K arrival counters
  // one block: compact the rows whose weight is non-zero into one-token items
  __shared__ int32_t base;
  if (threadIdx.x == 0) base = 0;
  __syncthreads();
  for (int i0 = 0; i0 < n; i0 += blockDim.x) {
    const int i = i0 + threadIdx.x;
    const bool on = i < n && w[i] != 0.f;
    const uint32_t bal = __ballot_sync(0xffffffffu, on);
    const int lane = threadIdx.x & 31;
    int wbase = 0;
    if (lane == 0 && bal) wbase = atomicAdd(&base, __popc(bal));
    wbase = __shfl_sync(0xffffffffu, wbase, 0);
    if (on) {
      const int j = wbase + __popc(bal & ((1u << lane) - 1u));
      Item it;
      it.p_guq = tab[4 * (int64_t)i + 0];
      it.p_gus = tab[4 * (int64_t)i + 1];
      it.p_dnq = tab[4 * (int64_t)i + 2];
      it.p_dns = tab[4 * (int64_t)i + 3];
      it.slot = 0;
      it.start = j;
      it.ntok = 1;
      it._pad = i;
      items[j] = it;
      pos[j] = i;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    *n_items = base;
    job_next[0] = 0;
    job_next[1] = 0;
  }
}

// Shared expert (Qwen3-Next): one warp per token computes the gate logit x[t] . wg (fp32 FMA chain
// over the columns lane*8 + 256*i + j, xor butterfly, rounded to the activation type as F.linear
// returns it) and the combine weight sigmoid(logit) in fp32; the first threads write the work items
// (consecutive tokens, nt per item) of the single shared record.
template <typename AT>
__global__ void __launch_bounds__(256) shared_gate_kernel(const AT* __restrict__ x, const AT* __restrict__ wg, int T,
                                                          int H, int nt, int64_t rec, LayoutOffs lo,
                                                          float* __restrict__ w, int32_t* __restrict__ pos,
                                                          Item* __restrict__ items, int32_t* __restrict__ n_items,
                                                          int32_t* __restrict__ job_next, int32_t* __restrict__ cnt,
                                                          int cnt_n) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gtid = blockIdx.x * blockDim.x + threadIdx.x;
  for (int i = gtid; i < cnt_n; i += gridDim.x * blockDim.x) cnt[i] = 0;  // split-K arrival counters
  const int ni = (T + nt - 1) / nt;
  if (gtid < ni) {
    Item it;
    it.p_guq = rec + lo.gu_q;
    it.p_gus = rec + lo.gu_s;
    it.p_dnq = rec + lo.dn_q;
    it.p_dns = rec + lo.dn_s;
    it.slot = 0;
    it.start = gtid * nt;
    it.ntok = min(nt, T - gtid * nt);
    it._pad = 0;
    items[gtid] = it;
  }
  if (gtid == 0) {
    *n_items = ni;
    job_next[0] = 0;
    job_next[1] = 0;
  }
  const int t = blockIdx.x * 8 + warp;
  if (t >= T) return;
  const AT* xr = x + (int64_t)t * H;
  float acc = 0.f;
  for (int c = lane * 8; c < H; c += 256) {
    const uint4 wv = __ldg(reinterpret_cast<const uint4*>(wg + c));
    const uint4 xv = __ldg(reinterpret_cast<const uint4*>(xr + c));
    const AT* wa = reinterpret_cast<const AT*>(&wv);
    const AT* xa = reinterpret_cast<const AT*>(&xv);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc = fmaf(to_f32<AT>(xa[i]), to_f32<AT>(wa[i]), acc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) {
    const float g = to_f32<AT>(from_f32<AT>(acc));
    w[t] = 1.f / (1.f + expf(-g));
    pos[t] = t;
  }
}

}  // namespace

namespace moeb200 {
// Phase mark of the measurement hooks (moeb200_trace_begin/end) on the stream, when tracing.
cudaError_t trace_mark(int which, cudaStream_t s) {
  if (!g_tracing) return cudaSuccess;
  if (which == 0) {
    if (g_trace_used == g_trace_pool.size()) {
      TraceRec r{};
      for (auto& e : r.ev) {
        cudaError_t err = cudaEventCreate(&e);
        if (err != cudaSuccess) return err;
      }
      g_trace_pool.push_back(r);
    }
    ++g_trace_used;
  }
  return cudaEventRecord(g_trace_pool[g_trace_used - 1].ev[which], s);
}

// SM count of the current device (cached per device).
int num_sms_cached() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lk(mu);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

// Records an error message for moeb200_last_error from other translation units of the library.
int set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  g_err_code = code;
  return code;
}
}  // namespace moeb200

extern "C" {

const char* moeb200_version(void) { return "moeb200 0.1 (sm_100a)"; }

int moeb200_last_error(char* buf, size_t n) {
  if (buf && n) {
    strncpy(buf, g_err.c_str(), n - 1);
    buf[n - 1] = '\0';
  }
  return g_err_code;
}

int moeb200_num_sms(void) { return num_sms_cached(); }

int moeb200_set_path(int32_t path) {
  if (path < 0 || path > 4)
    return fail(MOEB200_ERR_INVALID,
                "set_path: path must be 0 (auto), 1 (GEMV), 2 (GEMM), 3 (fused decode) or 4 (warp-streamed GEMV)");
  g_path = path;
  return MOEB200_OK;
}

int moeb200_set_item_tokens(int32_t nt) {
  if (nt != 0 && nt != 8 && nt != 16) return fail(MOEB200_ERR_INVALID, "set_item_tokens: 0 (automatic), 8 or 16");
  g_item_tokens = nt;
  return MOEB200_OK;
}

int moeb200_path_used(void) { return g_last_path; }

int moeb200_trace_begin(void) {
  g_tracing = true;
  g_trace_used = 0;
  return MOEB200_OK;
}

int moeb200_trace_end(float* up_ms, float* down_ms, int32_t* calls) {
  g_tracing = false;
  float up = 0.f, dn = 0.f;
  for (size_t i = 0; i < g_trace_used; ++i) {
    const TraceRec& r = g_trace_pool[i];
    CUDA_TRY(cudaEventSynchronize(r.ev[2]));
    float a = 0.f, b = 0.f;
    CUDA_TRY(cudaEventElapsedTime(&a, r.ev[0], r.ev[1]));
    CUDA_TRY(cudaEventElapsedTime(&b, r.ev[1], r.ev[2]));
    up += a;
    dn += b;
  }
  if (up_ms) *up_ms = up;
  if (down_ms) *down_ms = dn;
  if (calls) *calls = (int32_t)g_trace_used;
  g_trace_used = 0;
  return MOEB200_OK;
}

size_t moeb200_router_workspace(int32_t T, int32_t E) {
  Carve c(nullptr);
  c.take<WsHeader>(1);
  c.take<float>((size_t)T * E);
  return c.off;
}

namespace {
int router_impl(const void* h, const void* wr, const float* bias, int32_t act_type, int32_t T, int32_t H, int32_t E,
                int32_t k, int32_t renorm, float* probs, float* w, int64_t* idx, float* logits_out,
                const moeb200_policy* policy, uint8_t* level, uint8_t* skip, void* ws, size_t ws_bytes, void* stream,
                int shared_level) {
  if (!h || !wr || !w || !idx) return fail(MOEB200_ERR_INVALID, "router: null pointer");
  if (T <= 0 || H <= 0 || E <= 0 || k <= 0 || k > 32 || k > E || E > 1024)
    return fail(MOEB200_ERR_INVALID, "router: bad sizes T=%d H=%d E=%d k=%d (k <= 32, E <= 1024)", T, H, E, k);
  if (act_type != MOEB200_F16 && act_type != MOEB200_BF16 && act_type != MOEB200_F32)
    return fail(MOEB200_ERR_INVALID, "router: activation type must be F16, BF16 or F32");
  if (H % (act_type == MOEB200_F32 ? 4 : 8)) return fail(MOEB200_ERR_UNSUPPORTED, "router: H must be a multiple of 8");
  if (policy && !level) return fail(MOEB200_ERR_INVALID, "router: policy given without a level output");
  const int cols = shared_level >= 0 ? E + 1 : E;  // logit columns
  if (ws_bytes < moeb200_router_workspace(T, cols)) return fail(MOEB200_ERR_WORKSPACE, "router: workspace too small");
  Carve c(ws);
  WsHeader* hdr = c.take<WsHeader>(1);
  (void)hdr;
  float* logits = c.take<float>((size_t)T * cols);
  if (logits_out) logits = logits_out;
  PolicyDev pd{};
  if (policy) pd = {policy->mode, policy->t1, policy->t_mid, policy->t2, policy->thr};
  CUDA_TRY(launch_router(h, wr, bias, act_type, T, H, E, k, renorm, logits, probs, w, idx, policy ? &pd : nullptr,
                         level, skip, static_cast<cudaStream_t>(stream), shared_level));
  return MOEB200_OK;
}
}  // namespace

int moeb200_router(const void* h, const void* wr, const float* bias, int32_t act_type, int32_t T, int32_t H, int32_t E,
                   int32_t k, int32_t renorm, float* probs, float* w, int64_t* idx, float* logits_out,
                   const moeb200_policy* policy, uint8_t* level, uint8_t* skip, void* ws, size_t ws_bytes,
                   void* stream) {
  return router_impl(h, wr, bias, act_type, T, H, E, k, renorm, probs, w, idx, logits_out, policy, level, skip, ws,
                     ws_bytes, stream, -1);
}

int moeb200_router_shared(const void* h, const void* wr, const float* bias, int32_t act_type, int32_t T, int32_t H,
                          int32_t E, int32_t k, int32_t renorm, int32_t shared_level, float* probs, float* w,
                          int64_t* idx, float* logits_out, const moeb200_policy* policy, uint8_t* level,
                          uint8_t* skip, void* ws, size_t ws_bytes, void* stream) {
  if (shared_level < 0 || shared_level > 2) return fail(MOEB200_ERR_INVALID, "router_shared: shared_level must be 0, 1 or 2");
  if (k + 1 > 32) return fail(MOEB200_ERR_INVALID, "router_shared: k + 1 must be at most 32");
  if (E + 1 > 1024) return fail(MOEB200_ERR_INVALID, "router_shared: E + 1 must be at most 1024");
  return router_impl(h, wr, bias, act_type, T, H, E, k, renorm, probs, w, idx, logits_out, policy, level, skip, ws,
                     ws_bytes, stream, shared_level);
}

int moeb200_levels(const float* w, int32_t T, int32_t k, const moeb200_policy* policy, uint8_t* level, uint8_t* skip,
                   void* stream) {
  if (!w || !policy || !level) return fail(MOEB200_ERR_INVALID, "levels: null pointer");
  if (T <= 0 || k <= 0 || k > 32) return fail(MOEB200_ERR_INVALID, "levels: bad sizes T=%d k=%d", T, k);
  if (policy->mode < 0 || policy->mode > 3) return fail(MOEB200_ERR_INVALID, "levels: unknown mode %d", policy->mode);
  PolicyDev pd{policy->mode, policy->t1, policy->t_mid, policy->t2, policy->thr};
  CUDA_TRY(launch_levels(w, T, k, pd, level, skip, static_cast<cudaStream_t>(stream)));
  return MOEB200_OK;
}

int moeb200_levels_vote(const int64_t* idx, uint8_t* level, const uint8_t* skip, int32_t T, int32_t k, int32_t E,
                        double hi_vote, void* stream) {
  if (!idx || !level) return fail(MOEB200_ERR_INVALID, "levels_vote: null pointer");
  if (T <= 0 || k <= 0 || k > 32 || (int64_t)T * k >= (1ll << 30))
    return fail(MOEB200_ERR_INVALID, "levels_vote: bad sizes T=%d k=%d", T, k);
  if (E <= 0 || E > 16384) return fail(MOEB200_ERR_INVALID, "levels_vote: E=%d outside [1, 16384]", E);
  if (!(hi_vote >= 0.0 && hi_vote <= 1.0)) return fail(MOEB200_ERR_INVALID, "levels_vote: hi_vote outside [0, 1]");
  CUDA_TRY(launch_levels_vote(idx, level, skip, T * k, E, hi_vote, static_cast<cudaStream_t>(stream)));
  return MOEB200_OK;
}

size_t moeb200_dispatch_workspace(int32_t T, int32_t k, int32_t E, int32_t P) {
  const int n = T * k;
  const int nblk = (n + kDispBlock - 1) / kDispBlock;
  Carve c(nullptr);
  c.take<WsHeader>(1);
  c.take<int32_t>((size_t)nblk * E * P);
  c.take<int32_t>((size_t)nblk * E);
  c.take<int32_t>(n);
  c.take<int32_t>(n);
  c.take<int32_t>((size_t)E * P);
  c.take<int32_t>(E);
  return c.off;
}

int moeb200_dispatch(const int64_t* idx, const uint8_t* level, const uint8_t* skip, int32_t T, int32_t k, int32_t E,
                     int32_t P, int32_t* counts_e, int32_t* pos_e, int32_t* counts_k, int32_t* pos_k, int32_t* n_kept,
                     void* ws, size_t ws_bytes, void* stream) {
  if (!idx || !counts_e || !pos_e || !counts_k || !pos_k) return fail(MOEB200_ERR_INVALID, "dispatch: null pointer");
  if (T <= 0 || k <= 0 || E <= 0 || P <= 0 || P > 4 || (int64_t)E * P > kMaxKeys || (int64_t)T * k >= (1ll << 30))
    return fail(MOEB200_ERR_INVALID, "dispatch: bad sizes T=%d k=%d E=%d P=%d (E*P <= %d)", T, k, E, P, kMaxKeys);
  if (ws_bytes < moeb200_dispatch_workspace(T, k, E, P)) return fail(MOEB200_ERR_WORKSPACE, "dispatch: workspace too small");
  const int n = T * k;
  DispatchParams dp{};
  Carve c(ws);
  WsHeader* hdr = c.take<WsHeader>(1);
  dp.e_lo = 0;
  dp.e_hi = E;
  dp.nblk = (n + kDispBlock - 1) / kDispBlock;
  dp.blk_k = c.take<int32_t>((size_t)dp.nblk * E * P);
  dp.blk_e = c.take<int32_t>((size_t)dp.nblk * E);
  dp.rank_k = c.take<int32_t>(n);
  dp.rank_e = c.take<int32_t>(n);
  dp.offs_k = c.take<int32_t>((size_t)E * P);
  dp.offs_e = c.take<int32_t>(E);
  dp.idx = idx;
  dp.level = level;
  dp.skip = skip;
  dp.T = T;
  dp.k = k;
  dp.E = E;
  dp.P = P;
  dp.nt = 8;
  dp.counts_e = counts_e;
  dp.pos_e = pos_e;
  dp.counts_k = counts_k;
  dp.pos_k = pos_k;
  dp.n_kept = n_kept;
  dp.status = &hdr->status;
  CUDA_TRY(launch_dispatch(dp, static_cast<cudaStream_t>(stream)));
  return MOEB200_OK;
}

size_t moeb200_grouped_ffn_workspace(const moeb200_layout* layout, int32_t n) {
  if (!layout || n <= 0) return 0;
  Carve c(nullptr);
  c.take<WsHeader>(1);
  c.take<Item>(n);
  c.take<int32_t>(n);
  c.take<uint8_t>((size_t)n * layout->inter * 2);
  c.take<float>((size_t)table_split_slices(n, layout->inter) * split_rows(n) * 2 * layout->inter);
  c.take<int32_t>(split_cnt_ints(n, layout->inter));
  c.take<uint8_t>((size_t)kTmapSlots * kGemvMaxGrid * 128);
  c.take<float>((size_t)layout->hidden);
  return c.off;
}

int moeb200_grouped_ffn(const moeb200_layout* layout, const int64_t* tab, const float* w, int32_t n, const void* x,
                        int32_t act_type, void* out, void* ws, size_t ws_bytes, void* stream) {
  if (!layout || !tab || !w || !x || !out || !ws) return fail(MOEB200_ERR_INVALID, "grouped_ffn: null pointer");
  if (n <= 0 || n > 4096) return fail(MOEB200_ERR_INVALID, "grouped_ffn: n=%d out of range", n);
  if (act_type != MOEB200_F16 && act_type != MOEB200_BF16)
    return fail(MOEB200_ERR_UNSUPPORTED, "grouped_ffn: activations must be F16 or BF16 (tensor-core operands)");
  const int H = layout->hidden, I = layout->inter;
  int rc = check_shapes(H, I);
  if (rc) return rc;
  rc = check_layout(*layout, H, I);
  if (rc) return rc;
  if (ws_bytes < moeb200_grouped_ffn_workspace(layout, n))
    return fail(MOEB200_ERR_WORKSPACE, "grouped_ffn: workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Carve c(ws);
  WsHeader* hdr = c.take<WsHeader>(1);
  Item* items = c.take<Item>(n);
  int32_t* pos = c.take<int32_t>(n);
  uint8_t* hbuf = c.take<uint8_t>((size_t)n * I * 2);
  const int slices = table_split_slices(n, I);
  float* pre = c.take<float>((size_t)slices * split_rows(n) * 2 * I);
  int32_t* cnt = c.take<int32_t>(split_cnt_ints(n, I));
  uint8_t* tmaps = c.take<uint8_t>((size_t)kTmapSlots * kGemvMaxGrid * 128);
  float* acc = c.take<float>((size_t)H);
  table_items_kernel<<<1, 256, 0, s>>>(tab, w, n, items, &hdr->n_items, pos, hdr->job_next, cnt, split_cnt_ints(n, I));
  CUDA_TRY(cudaGetLastError());
  GemvParams gp{};
  gp.items = items;
  gp.n_items = &hdr->n_items;
  gp.pos = pos;
  gp.wflat = w;
  gp.k = n;
  gp.H = H;
  gp.I = I;
  gp.T = 1;
  gp.x = x;
  gp.h = hbuf;
  gp.pre = pre;
  gp.tile_cnt = cnt;
  gp.pre_rows = split_rows(n);
  gp.pre_slices = slices;
  gp.tmap_ws = tmaps;
  gp.acc = acc;
  gp.status = &hdr->status;
  gp.job_next = hdr->job_next;
  gp.lay[0] = to_dev(*layout);
  gp.zero_acc = 1;
  return run_expert_phases(gp, layout, 1, act_type, n, n, 8, s, out, /*add=*/1);
}

size_t moeb200_experts_workspace(const moeb200_expert_table* ex, int32_t T, int32_t k) {
  if (!ex || ex->n_prec <= 0) return 0;
  return carve_forward(nullptr, T, k, ex->num_experts, ex->n_prec, ex->layout[0].hidden, ex->layout[0].inter, MOEB200_F16)
      .bytes;
}

namespace {
// Shared body of moeb200_experts_forward (out in act_type) and moeb200_experts_forward_part
// (part: fp32 partial sums over the experts [e_lo, e_hi), written straight by the down phase).
int experts_forward_impl(const moeb200_expert_table* ex, int32_t e_lo, int32_t e_hi, const void* x, int32_t act_type,
                         int32_t T, const int64_t* idx, const float* w, int32_t k, const uint8_t* level,
                         const uint8_t* skip, void* out, float* part, int32_t* miss, void* ws, size_t ws_bytes,
                         void* stream) {
  if (!ex || !ex->table || !x || !idx || !w || (!out && !part) || !ws)
    return fail(MOEB200_ERR_INVALID, "experts_forward: null pointer");
  const int P = ex->n_prec, E = ex->num_experts;
  if (P <= 0 || P > 4 || E <= 0 || (int64_t)E * P > kMaxKeys)
    return fail(MOEB200_ERR_INVALID, "experts_forward: bad table (P=%d, E=%d, E*P <= %d)", P, E, kMaxKeys);
  if (e_lo < 0 || e_hi > E || e_lo >= e_hi)
    return fail(MOEB200_ERR_INVALID, "experts_forward: bad expert range [%d, %d) of %d", e_lo, e_hi, E);
  if (T <= 0 || k <= 0 || k > 32 || (int64_t)T * k >= (1ll << 30))
    return fail(MOEB200_ERR_INVALID, "experts_forward: bad sizes T=%d k=%d", T, k);
  if (act_type != MOEB200_F16 && act_type != MOEB200_BF16)
    return fail(MOEB200_ERR_UNSUPPORTED, "experts_forward: activations must be F16 or BF16");
  const int H = ex->layout[0].hidden, I = ex->layout[0].inter;
  int rc = check_shapes(H, I);
  if (rc) return rc;
  for (int p = 0; p < P; ++p) {
    rc = check_layout(ex->layout[p], H, I);
    if (rc) return rc;
  }
  ForwardWs fw = carve_forward(nullptr, T, k, E, P, H, I, act_type);
  if (ws_bytes < fw.bytes) return fail(MOEB200_ERR_WORKSPACE, "experts_forward: workspace too small (%zu < %zu)", ws_bytes, fw.bytes);
  fw = carve_forward(ws, T, k, E, P, H, I, act_type);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int n = T * k;
  // tcgen05 GEMM when experts see many tokens (prefill), else the grouped GEMV. The switch sits at
  // 40 routed pairs per expert on average (measured, config 1 shapes: GEMV 1.44x faster at 16 pairs
  // per expert, 1.13x at 32, the GEMM 1.22x faster at 64); under expert parallelism n counts every
  // rank's tokens, so the rule sees the pairs per local expert.
  const bool gemm_ok = (H % 128 == 0) && (I % 128 == 0);
  bool gemm = g_path == 2 || (g_path == 0 && (int64_t)n >= kGemmPairsPerExpert * E);
  if (gemm && !gemm_ok) {
    if (g_path == 2) return fail(MOEB200_ERR_UNSUPPORTED, "GEMM path needs H and I multiples of 128 (H=%d, I=%d)", H, I);
    gemm = false;
  }
  const bool dec_ok = ex->tma_base != 0 && ex->tma_base % 4096 == 0 && decode_supported(ex->layout, P, act_type, H, I);
  if (g_path == 3 && !dec_ok)
    return fail(MOEB200_ERR_UNSUPPORTED, "decode path: these record layouts or shapes are not supported by the fused "
                                         "decode kernel");
  // the fused decode kernel is taken only when asked for (path 3): measured slower than the
  // two-launch grouped GEMV on every decode workload of the build's configs so far
  const bool decode = !gemm && g_path == 3;
  // warp-streamed GEMV: items of <= 8 pairs; x rows are staged with 16-byte bulk copies
  const bool ws_ok = ws_supported(ex->layout, P, act_type, H, I, 8) && reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
                     ex->tma_base != 0 && ex->tma_base % 4096 == 0;
  if (g_path == 4 && !ws_ok)
    return fail(MOEB200_ERR_UNSUPPORTED, "warp-streamed GEMV: these record layouts, shapes or the x alignment are "
                                         "not supported");
  // automatic path: the warp-streamed GEMV for calls of up to 8 tokens (measured, 16 layers of
  // config 1, against the CTA-pipeline GEMV: T = 2 2,440 / 2,100 tokens/s, T = 4 3,649 / 3,414,
  // T = 8 5,449 / 5,434)
  const bool streamed = !gemm && !decode && (g_path == 4 || (g_path == 0 && T <= 8 && ws_ok));
  // (the warp-streamed GEMV stages at most min(8, T) activation rows per item)
  const int nt = gemm ? 128 : decode ? 8 : streamed ? std::min(8, T) : g_item_tokens ? g_item_tokens : (T >= 64 ? 16 : 8);
  g_last_path = gemm ? 2 : decode ? 3 : streamed ? 4 : 1;
  // upper bound on items: every key splits into ceil(c / nt) items
  const int64_t max_items = std::min<int64_t>(n, (int64_t)(n + nt - 1) / nt + (int64_t)(e_hi - e_lo) * P);
  DispatchParams dp{};
  dp.idx = idx;
  dp.level = level;
  dp.skip = skip;
  dp.T = T;
  dp.k = k;
  dp.E = E;
  dp.P = P;
  dp.e_lo = e_lo;
  dp.e_hi = e_hi;
  dp.nblk = (n + kDispBlock - 1) / kDispBlock;
  dp.nt = nt;
  dp.counts_e = fw.counts_e;
  dp.pos_e = fw.pos_e;
  dp.counts_k = fw.counts_k;
  dp.offs_k = fw.offs_k;
  dp.offs_e = fw.offs_e;
  dp.pos_k = fw.pos_k;
  dp.n_kept = &fw.hdr->n_kept;
  dp.blk_k = fw.blk_k;
  dp.blk_e = fw.blk_e;
  dp.rank_k = fw.rank_k;
  dp.rank_e = fw.rank_e;
  dp.items = fw.items;
  dp.n_items = &fw.hdr->n_items;
  dp.table = ex->table;
  for (int p = 0; p < P; ++p) {
    const moeb200_layout& L = ex->layout[p];
    dp.offs[p] = {L.off_gu_q, is_int(L.wtype) ? L.off_gu_s : 0, L.off_dn_q, is_int(L.wtype) ? L.off_dn_s : 0};
  }
  dp.miss = miss ? miss : &fw.hdr->miss;
  dp.status = &fw.hdr->status;
  dp.job_next = fw.hdr->job_next;
  dp.zero_cnt = fw.cnt;
  dp.zero_n = decode ? (int)decode_cnt_ints(max_items, H) : split_cnt_ints(n, I);
  dp.slot_items = decode ? fw.cnt + kDecSlotItems : nullptr;
  CUDA_TRY(launch_dispatch(dp, s));
  if (decode) {
    DecodeParams q{};
    q.items = fw.items;
    q.n_items = &fw.hdr->n_items;
    q.pos = fw.pos_k;
    q.wflat = w;
    q.k = k;
    q.H = H;
    q.I = I;
    q.T = T;
    q.x = x;
    q.h = fw.h;
    q.acc = part ? part : fw.acc;
    q.out = part ? nullptr : out;
    q.add = 0;
    q.max_items = (int)max_items;
    q.status = &fw.hdr->status;
    q.ctr = fw.cnt;
    q.updone = fw.cnt + kDecUpdone;
    q.slot_items = fw.cnt + kDecSlotItems;
    q.nprec = P;
    q.tma_base = ex->tma_base;
    for (int p = 0; p < P; ++p) q.lay[p] = to_dev(ex->layout[p]);
    const int64_t units = max_items * (I / 8 + H / 16);
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(num_sms_cached(), units));
    CUDA_TRY(trace_mark(0, s));
    CUDA_TRY(launch_decode(q, ex->layout, P, act_type, grid, s));
    CUDA_TRY(trace_mark(1, s));
    CUDA_TRY(trace_mark(2, s));
    return MOEB200_OK;
  }
  GemvParams gp{};
  gp.items = fw.items;
  gp.n_items = &fw.hdr->n_items;
  gp.pos = fw.pos_k;
  gp.wflat = w;
  gp.k = k;
  gp.H = H;
  gp.I = I;
  gp.T = T;
  gp.x = x;
  gp.h = fw.h;
  gp.pre = fw.pre;
  gp.tile_cnt = fw.cnt;
  gp.pre_rows = split_rows(n);
  gp.tmap_ws = fw.tmaps;
  gp.acc = part ? part : fw.acc;
  gp.status = &fw.hdr->status;
  gp.job_next = fw.hdr->job_next;
  for (int p = 0; p < P; ++p) gp.lay[p] = to_dev(ex->layout[p]);
  gp.zero_acc = 1;
  gp.tma_base = ex->tma_base;
  return run_expert_phases(gp, ex->layout, P, act_type, (int)max_items, n, nt, s, part ? nullptr : out, /*add=*/0,
                           gemm, streamed);
}
}  // namespace

int moeb200_experts_forward(const moeb200_expert_table* ex, const void* x, int32_t act_type, int32_t T,
                            const int64_t* idx, const float* w, int32_t k, const uint8_t* level, const uint8_t* skip,
                            void* out, int32_t* miss, void* ws, size_t ws_bytes, void* stream) {
  if (!out) return fail(MOEB200_ERR_INVALID, "experts_forward: null pointer");
  return experts_forward_impl(ex, 0, ex ? ex->num_experts : 0, x, act_type, T, idx, w, k, level, skip, out, nullptr,
                              miss, ws, ws_bytes, stream);
}

int moeb200_experts_forward_part(const moeb200_expert_table* ex, int32_t e_lo, int32_t e_hi, const void* x,
                                 int32_t act_type, int32_t T, const int64_t* idx, const float* w, int32_t k,
                                 const uint8_t* level, const uint8_t* skip, float* part, int32_t* miss, void* ws,
                                 size_t ws_bytes, void* stream) {
  if (!part) return fail(MOEB200_ERR_INVALID, "experts_forward_part: null pointer");
  return experts_forward_impl(ex, e_lo, e_hi, x, act_type, T, idx, w, k, level, skip, nullptr, part, miss, ws,
                              ws_bytes, stream);
}

int moeb200_combine_parts(const float* parts, int32_t G, int64_t n, int32_t act_type, void* out, int32_t add,
                          void* stream) {
  if (!parts || !out) return fail(MOEB200_ERR_INVALID, "combine_parts: null pointer");
  if (G <= 0 || G > 64 || n <= 0) return fail(MOEB200_ERR_INVALID, "combine_parts: bad sizes G=%d n=%lld", G, (long long)n);
  if (act_type != MOEB200_F16 && act_type != MOEB200_BF16 && act_type != MOEB200_F32)
    return fail(MOEB200_ERR_UNSUPPORTED, "combine_parts: output must be F32, F16 or BF16");
  CUDA_TRY(launch_combine_parts(parts, G, n, act_type, out, add, static_cast<cudaStream_t>(stream)));
  return MOEB200_OK;
}

size_t moeb200_shared_expert_workspace(const moeb200_layout* layout, int32_t T) {
  if (!layout || T <= 0) return 0;
  Carve c(nullptr);
  c.take<WsHeader>(1);
  c.take<Item>(T);
  c.take<int32_t>(T);
  c.take<float>(T);
  c.take<uint8_t>((size_t)T * layout->inter * 2);
  c.take<float>(split_pre_floats(T, layout->inter));
  c.take<int32_t>(split_cnt_ints(T, layout->inter));
  c.take<uint8_t>((size_t)kTmapSlots * kGemvMaxGrid * 128);
  c.take<float>((size_t)T * layout->hidden);
  return c.off;
}

int moeb200_shared_expert(const moeb200_layout* layout, const void* record, const void* wg, const void* x,
                          int32_t act_type, int32_t T, void* out, int32_t add, void* ws, size_t ws_bytes,
                          void* stream) {
  if (!layout || !record || !wg || !x || !out || !ws) return fail(MOEB200_ERR_INVALID, "shared_expert: null pointer");
  if (T <= 0 || T >= (1 << 24)) return fail(MOEB200_ERR_INVALID, "shared_expert: bad T=%d", T);
  if (act_type != MOEB200_F16 && act_type != MOEB200_BF16)
    return fail(MOEB200_ERR_UNSUPPORTED, "shared_expert: activations must be F16 or BF16");
  const int H = layout->hidden, I = layout->inter;
  int rc = check_shapes(H, I);
  if (rc) return rc;
  rc = check_layout(*layout, H, I);
  if (rc) return rc;
  if (reinterpret_cast<uintptr_t>(record) % 256) return fail(MOEB200_ERR_INVALID, "shared_expert: record must be 256-byte aligned");
  if (ws_bytes < moeb200_shared_expert_workspace(layout, T))
    return fail(MOEB200_ERR_WORKSPACE, "shared_expert: workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool gemm_ok = (H % 128 == 0) && (I % 128 == 0);
  bool gemm = g_path == 2 || (g_path == 0 && T >= 64);
  if (gemm && !gemm_ok) {
    if (g_path == 2) return fail(MOEB200_ERR_UNSUPPORTED, "GEMM path needs H and I multiples of 128 (H=%d, I=%d)", H, I);
    gemm = false;
  }
  const int nt = gemm ? 128 : g_item_tokens ? g_item_tokens : (T >= 128 ? 16 : 8);
  Carve c(ws);
  WsHeader* hdr = c.take<WsHeader>(1);
  Item* items = c.take<Item>(T);
  int32_t* pos = c.take<int32_t>(T);
  float* wt = c.take<float>(T);
  uint8_t* hbuf = c.take<uint8_t>((size_t)T * I * 2);
  float* pre = c.take<float>(split_pre_floats(T, I));
  int32_t* cnt = c.take<int32_t>(split_cnt_ints(T, I));
  uint8_t* tmaps = c.take<uint8_t>((size_t)kTmapSlots * kGemvMaxGrid * 128);
  float* acc = c.take<float>((size_t)T * H);
  const LayoutOffs lo{layout->off_gu_q, is_int(layout->wtype) ? layout->off_gu_s : 0, layout->off_dn_q,
                      is_int(layout->wtype) ? layout->off_dn_s : 0};
  const int64_t rec = (int64_t)reinterpret_cast<uintptr_t>(record);
  const int grid = (T + 7) / 8;
  if (act_type == MOEB200_BF16)
    shared_gate_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x),
                                                           static_cast<const __nv_bfloat16*>(wg), T, H, nt, rec, lo, wt,
                                                           pos, items, &hdr->n_items, hdr->job_next, cnt,
                                                           split_cnt_ints(T, I));
  else
    shared_gate_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(x), static_cast<const __half*>(wg), T, H,
                                                    nt, rec, lo, wt, pos, items, &hdr->n_items, hdr->job_next, cnt,
                                                    split_cnt_ints(T, I));
  CUDA_TRY(cudaGetLastError());
  GemvParams gp{};
  gp.items = items;
  gp.n_items = &hdr->n_items;
  gp.pos = pos;
  gp.wflat = wt;
  gp.k = 1;
  gp.H = H;
  gp.I = I;
  gp.T = T;
  gp.x = x;
  gp.h = hbuf;
  gp.pre = pre;
  gp.tile_cnt = cnt;
  gp.pre_rows = split_rows(T);
  gp.tmap_ws = tmaps;
  gp.acc = acc;
  gp.status = &hdr->status;
  gp.job_next = hdr->job_next;
  gp.lay[0] = to_dev(*layout);
  gp.zero_acc = 1;
  return run_expert_phases(gp, layout, 1, act_type, (T + nt - 1) / nt, T, nt, s, out, add ? 1 : 0, gemm);
}

int moeb200_check_workspace(void* ws, int32_t* status, void* stream) {
  if (!ws || !status) return fail(MOEB200_ERR_INVALID, "check_workspace: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  WsHeader* hdr = static_cast<WsHeader*>(ws);
  CUDA_TRY(cudaMemcpyAsync(status, &hdr->status, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
  CUDA_TRY(cudaStreamSynchronize(s));
  CUDA_TRY(cudaMemsetAsync(&hdr->status, 0, sizeof(int32_t), s));
  return MOEB200_OK;
}

}  // extern "C"
