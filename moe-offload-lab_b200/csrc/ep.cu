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

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>

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

// ---------------------------------------------------------------------------------------------------
// Peer-memory exchange (one process per GPU, buffers mapped into the peers with CUDA IPC).
//
// Every rank owns, in memory its peers can map: its packed exchange rows [T, row_bytes], its fp32
// partial sums over the gathered tokens [G*T, H], and flags int32 [2][G] (flags[0][s]: rank s's
// rows of call e are ready, flags[1][s]: rank s's partial sums of call e are ready). Per MoE layer:
//   pack (local) -> signal 0 (epoch += 1; flag[0][me] = epoch on every rank, release, system scope)
//   -> gather: wait flag[0][s] >= epoch, read rank s's rows over NVLink and unpack them at s*T
//   -> the owned experts write the local partial sums
//   -> signal 1 -> combine: wait flag[1][s] >= epoch, out[t] = sum over s (in rank order) of rank
//      s's partial row me*T + t, read over NVLink, cast once.
// Single buffers suffice: a rank packs call e+1 only after its combine of call e, which waited for
// every peer's partial sums of call e, so every peer had gathered call e; it overwrites its partial
// sums of call e+1 only after gathering call e+1, whose flags each peer raised after its combine
// of call e. Every wait is bounded: on timeout the status word is set and the kernel goes on.
// ---------------------------------------------------------------------------------------------------
namespace {

constexpr uint32_t kPeerSpin = 1u << 22;

__device__ __forceinline__ int ld_acquire_sys(const int32_t* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(int32_t* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Wait (bounded: `spin` polls) until *flag >= epoch; false and status set on timeout.
__device__ bool wait_flag(const int32_t* flag, int epoch, uint32_t spin, int32_t* status) {
  for (uint32_t i = 0; i < spin; ++i) {
    if (ld_acquire_sys(flag) >= epoch) return true;
    __nanosleep(64);
  }
  if (status) atomicExch(status, kDevTimeout);
  return false;
}

struct PeerArgs {
  const int64_t* rows;   // [G] each rank's packed rows
  const int64_t* parts;  // [G] each rank's partial sums
  const int64_t* flags;  // [G] each rank's flags
  int32_t* epoch;        // this rank's call counter
  int32_t* status;       // this rank's status word
  int32_t G, rank, T, H, k;
  uint32_t spin;         // polls per wait
};

// which == 0: epoch += 1 first. Then flag[which][rank] = epoch on every rank.
__global__ void ep_signal_kernel(PeerArgs a, int which) {
  __shared__ int ep;
  if (threadIdx.x == 0) {
    if (which == 0) *a.epoch += 1;
    ep = *a.epoch;
  }
  __syncthreads();
  __threadfence_system();  // this rank's writes of the previous kernels before the flags
  for (int s = threadIdx.x; s < a.G; s += blockDim.x) {
    int32_t* f = reinterpret_cast<int32_t*>(a.flags[s]) + which * a.G + a.rank;
    st_release_sys(f, ep);
  }
}

// Block (s, b): rank s's rows [b*rpb, (b+1)*rpb) -> the gathered arrays at token s*T + row.
__global__ void ep_gather_kernel(PeerArgs a, int xbytes, int rb, int rpb, uint8_t* __restrict__ x,
                                 int64_t* __restrict__ idx, float* __restrict__ w, uint8_t* __restrict__ level,
                                 uint8_t* __restrict__ skip) {
  const int s = blockIdx.x;
  __shared__ int ok;
  if (threadIdx.x == 0) {
    const int32_t* f = reinterpret_cast<const int32_t*>(a.flags[a.rank]) + s;
    ok = wait_flag(f, *a.epoch, a.spin, a.status);
  }
  __syncthreads();
  const uint8_t* src = reinterpret_cast<const uint8_t*>(a.rows[s]);
  const int k = a.k;
  for (int r = blockIdx.y * rpb; r < min(a.T, (blockIdx.y + 1) * rpb); ++r) {
    const uint8_t* row = src + (int64_t)r * rb;
    const int64_t t = (int64_t)s * a.T + r;
    const uint4* xs = reinterpret_cast<const uint4*>(row);
    uint4* xd = reinterpret_cast<uint4*>(x + t * xbytes);
    // peer data is read past the L1 (__ldcg): another GPU wrote it
    for (int i = threadIdx.x; i < xbytes / 16; i += blockDim.x) xd[i] = ok ? __ldcg(xs + i) : make_uint4(0, 0, 0, 0);
    const long long* ri = reinterpret_cast<const long long*>(row + xbytes);
    const float* rw = reinterpret_cast<const float*>(row + xbytes + 8 * k);
    const uint8_t* rl = row + xbytes + 12 * k;
    for (int j = threadIdx.x; j < k; j += blockDim.x) {
      const int64_t p = t * k + j;
      idx[p] = ok ? (int64_t)__ldcg(ri + j) : 0;
      w[p] = ok ? __ldcg(rw + j) : 0.f;
      const unsigned char lv = ok ? __ldcg(rl + j) : 0, sk = ok ? __ldcg(rl + k + j) : 1;
      if (level) level[p] = lv;
      if (skip) skip[p] = sk;  // a row that never arrived is dropped
    }
  }
}

// out[t] = act(sum over s in rank order of rank s's partial row rank*T + t) (+ out[t] when add).
template <typename AT>
__global__ void ep_combine_peers_kernel(PeerArgs a, AT* __restrict__ out, int add) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    const int32_t* f = reinterpret_cast<const int32_t*>(a.flags[a.rank]) + a.G;
    for (int s = 0; s < a.G; ++s) ok &= wait_flag(f + s, *a.epoch, a.spin, a.status);
  }
  __syncthreads();
  const int64_t n = (int64_t)a.T * a.H;
  const int64_t off = (int64_t)a.rank * a.T * a.H;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float v = 0.f;
    if (ok)
      for (int s = 0; s < a.G; ++s) v += __ldcg(reinterpret_cast<const float*>(a.parts[s]) + off + i);
    out[i] = from_f32<AT>(add ? to_f32<AT>(out[i]) + v : v);
  }
}

PeerArgs peer_args(const moeb200_peer_group* g) {
  PeerArgs a;
  a.rows = g->rows;
  a.parts = g->parts;
  a.flags = g->flags;
  a.epoch = g->epoch;
  a.status = g->status;
  a.G = g->G;
  a.rank = g->rank;
  a.T = g->T;
  a.H = g->H;
  a.k = g->k;
  a.spin = g->spin ? g->spin : kPeerSpin;
  return a;
}

int check_group(const moeb200_peer_group* g, const char* who) {
  if (!g || !g->rows || !g->parts || !g->flags || !g->epoch)
    return set_error(MOEB200_ERR_INVALID, "%s: incomplete peer group", who);
  if (g->G <= 0 || g->G > 64 || g->rank < 0 || g->rank >= g->G || g->T <= 0 || g->H <= 0 || g->k <= 0 || g->k > 32)
    return set_error(MOEB200_ERR_INVALID, "%s: bad peer group sizes", who);
  return MOEB200_OK;
}

}  // namespace

extern "C" {

int moeb200_peer_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return set_error(MOEB200_ERR_INVALID, "peer_alloc: bad arguments");
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return set_error(MOEB200_ERR_CUDA, "peer_alloc: %s", cudaGetErrorString(e));
  e = cudaMemset(*ptr, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), *ptr);
  if (e != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return set_error(MOEB200_ERR_CUDA, "peer_alloc: %s", cudaGetErrorString(e));
  }
  return MOEB200_OK;
}

int moeb200_peer_open(const void* handle, void** ptr) {
  if (!ptr || !handle) return set_error(MOEB200_ERR_INVALID, "peer_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_error(MOEB200_ERR_CUDA, "peer_open: %s", cudaGetErrorString(e));
  return MOEB200_OK;
}

int moeb200_peer_close(void* ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return set_error(MOEB200_ERR_CUDA, "peer_close: %s", cudaGetErrorString(e));
  return MOEB200_OK;
}

int moeb200_peer_free(void* ptr) {
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return set_error(MOEB200_ERR_CUDA, "peer_free: %s", cudaGetErrorString(e));
  return MOEB200_OK;
}

int moeb200_ep_signal(const moeb200_peer_group* g, int32_t which, void* stream) {
  int rc = check_group(g, "ep_signal");
  if (rc) return rc;
  if (which != 0 && which != 1) return set_error(MOEB200_ERR_INVALID, "ep_signal: which must be 0 (rows) or 1 (parts)");
  ep_signal_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(peer_args(g), which);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(MOEB200_ERR_CUDA, "ep_signal: %s", cudaGetErrorString(e));
  return MOEB200_OK;
}

int moeb200_ep_gather(const moeb200_peer_group* g, int32_t act_type, void* x, int64_t* idx, float* w, uint8_t* level,
                      uint8_t* skip, void* stream) {
  int rc = check_group(g, "ep_gather");
  if (rc) return rc;
  rc = check_args(g->T, g->H, g->k, act_type, "ep_gather");
  if (rc) return rc;
  if (!x || !idx || !w) return set_error(MOEB200_ERR_INVALID, "ep_gather: null pointer");
  const int rpb = 4;
  const dim3 grid(g->G, (g->T + rpb - 1) / rpb);
  ep_gather_kernel<<<grid, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      peer_args(g), g->H * elem_bytes(act_type), (int)row_bytes(g->H, g->k, act_type), rpb, static_cast<uint8_t*>(x),
      idx, w, level, skip);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(MOEB200_ERR_CUDA, "ep_gather: %s", cudaGetErrorString(e));
  return MOEB200_OK;
}

int moeb200_ep_combine_peers(const moeb200_peer_group* g, int32_t act_type, void* out, int32_t add, void* stream) {
  int rc = check_group(g, "ep_combine_peers");
  if (rc) return rc;
  if (!out) return set_error(MOEB200_ERR_INVALID, "ep_combine_peers: null pointer");
  const int64_t n = (int64_t)g->T * g->H;
  const int grid = (int)std::min<int64_t>((n + 255) / 256, 148 * 4);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const PeerArgs a = peer_args(g);
  if (act_type == MOEB200_BF16)
    ep_combine_peers_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(a, static_cast<__nv_bfloat16*>(out), add);
  else if (act_type == MOEB200_F16)
    ep_combine_peers_kernel<__half><<<grid, 256, 0, s>>>(a, static_cast<__half*>(out), add);
  else if (act_type == MOEB200_F32)
    ep_combine_peers_kernel<float><<<grid, 256, 0, s>>>(a, static_cast<float*>(out), add);
  else
    return set_error(MOEB200_ERR_UNSUPPORTED, "ep_combine_peers: output must be F32, F16 or BF16");
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(MOEB200_ERR_CUDA, "ep_combine_peers: %s", cudaGetErrorString(e));
  return MOEB200_OK;
}

}  // extern "C"
