// Dense int8 linear layers (the model's non-expert part in int8, moelab/denseq.py `QLinear`).
//
// Replaces the reference's Triton `_gemv8` (denseq.py:34-57, one token) and its prefill fallback
// (denseq.py:92-100: `dequantize` (quant.py:191-205) by row blocks + F.linear):
//
//   gemv    : y[t, o] = sum over groups g of s[o, g] * sum_{c in g} q[o, c] * x[t, c]   (fp32), cast to
//             the activation type, + bias[o]; for up to kDenseMaxT tokens at once.
//   dequant : w[o, c] = act(q[o, c]) * act(s[o, c / gs]) rounded once to the activation type -- the
//             values moelab's `dequantize(q, s, 8, dtype)` produces (q is exact in fp16 and bf16;
//             the fp16 scale is converted to the activation type first).
//
// The GEMV streams q once from HBM: a warp owns 4 rows and its lanes read 16 consecutive int8
// of each row per step (512 columns per warp step, fully coalesced), convert them once and multiply
// them with every token's activations (read through L1: all warps of the SM share them). A lane's
// 16 columns lie in one scale group (gs a multiple of 16), so its partial sum is scaled once.
#include <algorithm>

#include "common.cuh"

namespace moeb200 {

int set_error(int code, const char* fmt, ...);  // capi.cu: records the message for moeb200_last_error

namespace {

constexpr int kDenseMaxT = 8;   // tokens per GEMV call
constexpr int kRows = 4;  // rows per warp (8 measured slower for one token: half the warps in flight)
constexpr int kDenseThreads = 256;

template <typename AT>
__device__ __forceinline__ void x16(const AT* p, float (&f)[16]) {
  const uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
  const uint4 b = __ldg(reinterpret_cast<const uint4*>(p) + 1);
  const AT* ha = reinterpret_cast<const AT*>(&a);
  const AT* hb = reinterpret_cast<const AT*>(&b);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    f[i] = to_f32<AT>(ha[i]);
    f[8 + i] = to_f32<AT>(hb[i]);
  }
}

template <typename AT, int NT>
__global__ void __launch_bounds__(kDenseThreads) dense_gemv_kernel(const int8_t* __restrict__ q,
                                                                   const __half* __restrict__ s, int O, int K,
                                                                   int gs, const AT* __restrict__ x,
                                                                   const AT* __restrict__ bias, AT* __restrict__ y) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int o0 = (blockIdx.x * (kDenseThreads / 32) + warp) * kRows;
  if (o0 >= O) return;
  const int ng = K / gs;
  float acc[kRows][NT];
#pragma unroll
  for (int r = 0; r < kRows; ++r)
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
  for (int c = lane * 16; c < K; c += 512) {
    // the kRows rows' 16 int8 of this step (rows past O read row O-1 and are not stored)
    int4 raw[kRows];
#pragma unroll
    for (int r = 0; r < kRows; ++r)
      raw[r] = __ldcs(reinterpret_cast<const int4*>(q + (int64_t)min(o0 + r, O - 1) * K + c));
    float sc[kRows];
#pragma unroll
    for (int r = 0; r < kRows; ++r) sc[r] = __half2float(s[(int64_t)min(o0 + r, O - 1) * ng + c / gs]);
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      float xf[16];
      x16<AT>(x + (int64_t)t * K + c, xf);
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        const int8_t* qb = reinterpret_cast<const int8_t*>(&raw[r]);
        float part = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) part = fmaf((float)qb[i], xf[i], part);
        acc[r][t] = fmaf(sc[r], part, acc[r][t]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kRows; ++r)
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      float v = acc[r][t];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      acc[r][t] = v;
    }
  static_assert(kRows * NT <= 32, "one lane per (row, token) result");
  if (lane < kRows * NT) {
    const int r = lane / NT, t = lane % NT;
    float v = 0.f;
#pragma unroll
    for (int rr = 0; rr < kRows; ++rr)
#pragma unroll
      for (int tt = 0; tt < NT; ++tt)
        if (rr == r && tt == t) v = acc[rr][tt];
    const int o = o0 + r;
    if (o < O) {
      const AT yv = from_f32<AT>(v);
      // bias added in the activation type after the cast, as `y + bias.to(y.dtype)` does
      y[(int64_t)t * O + o] = bias ? from_f32<AT>(to_f32<AT>(yv) + to_f32<AT>(bias[o])) : yv;
    }
  }
}

template <typename AT>
__global__ void dense_dequant_kernel(const int8_t* __restrict__ q, const __half* __restrict__ s, int64_t n, int K,
                                     int gs, AT* __restrict__ w) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = i / K;
    const int c = (int)(i - o * K);
    const AT qv = from_f32<AT>((float)q[i]);                                       // exact (|q| <= 127)
    const AT sv = from_f32<AT>(__half2float(s[o * (K / gs) + c / gs]));            // scales.to(dtype)
    w[i] = from_f32<AT>(to_f32<AT>(qv) * to_f32<AT>(sv));  // one rounding of the exact product
  }
}

template <typename AT>
cudaError_t gemv_t(const int8_t* q, const __half* s, int O, int K, int gs, const void* x, int T, const void* bias,
                   void* y, cudaStream_t st) {
  const int rows_per_block = (kDenseThreads / 32) * kRows;
  const int grid = (O + rows_per_block - 1) / rows_per_block;
  const AT* xa = static_cast<const AT*>(x);
  const AT* ba = static_cast<const AT*>(bias);
  AT* ya = static_cast<AT*>(y);
  switch (T) {
#define MOEB200_DG(N) \
  case N: dense_gemv_kernel<AT, N><<<grid, kDenseThreads, 0, st>>>(q, s, O, K, gs, xa, ba, ya); break;
    MOEB200_DG(1) MOEB200_DG(2) MOEB200_DG(3) MOEB200_DG(4) MOEB200_DG(5) MOEB200_DG(6) MOEB200_DG(7) MOEB200_DG(8)
#undef MOEB200_DG
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace

}  // namespace moeb200

using namespace moeb200;

extern "C" {

int moeb200_dense_int8_gemv(const int8_t* q, const uint16_t* s, int32_t O, int32_t K, int32_t gs, const void* x,
                            int32_t act_type, int32_t T, const void* bias, void* y, void* stream) {
  if (!q || !s || !x || !y) return set_error(MOEB200_ERR_INVALID, "dense_int8_gemv: null pointer");
  if (O <= 0 || K <= 0 || T <= 0 || T > kDenseMaxT)
    return set_error(MOEB200_ERR_INVALID, "dense_int8_gemv: bad sizes O=%d K=%d T=%d (1 <= T <= %d)", O, K, T,
                     kDenseMaxT);
  if (gs <= 0 || gs % 16 || K % gs)
    return set_error(MOEB200_ERR_UNSUPPORTED, "dense_int8_gemv: group size %d must be a multiple of 16 dividing K=%d",
                     gs, K);
  if (act_type != MOEB200_F16 && act_type != MOEB200_BF16)
    return set_error(MOEB200_ERR_UNSUPPORTED, "dense_int8_gemv: activations must be F16 or BF16");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(x)) % 16)
    return set_error(MOEB200_ERR_INVALID, "dense_int8_gemv: q and x must be 16-byte aligned");
  const __half* sh = reinterpret_cast<const __half*>(s);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const cudaError_t e = act_type == MOEB200_BF16 ? gemv_t<__nv_bfloat16>(q, sh, O, K, gs, x, T, bias, y, st)
                                                 : gemv_t<__half>(q, sh, O, K, gs, x, T, bias, y, st);
  if (e != cudaSuccess) return set_error(MOEB200_ERR_CUDA, "dense_int8_gemv: %s", cudaGetErrorString(e));
  return MOEB200_OK;
}

int moeb200_dense_int8_dequant(const int8_t* q, const uint16_t* s, int32_t O, int32_t K, int32_t gs,
                               int32_t act_type, void* w, void* stream) {
  if (!q || !s || !w) return set_error(MOEB200_ERR_INVALID, "dense_int8_dequant: null pointer");
  if (O <= 0 || K <= 0 || gs <= 0 || K % gs)
    return set_error(MOEB200_ERR_INVALID, "dense_int8_dequant: bad sizes O=%d K=%d gs=%d", O, K, gs);
  if (act_type != MOEB200_F16 && act_type != MOEB200_BF16)
    return set_error(MOEB200_ERR_UNSUPPORTED, "dense_int8_dequant: output must be F16 or BF16");
  const int64_t n = (int64_t)O * K;
  const int grid = (int)std::min<int64_t>((n + 255) / 256, 148 * 32);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const __half* sh = reinterpret_cast<const __half*>(s);
  if (act_type == MOEB200_BF16)
    dense_dequant_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(q, sh, n, K, gs, static_cast<__nv_bfloat16*>(w));
  else
    dense_dequant_kernel<__half><<<grid, 256, 0, st>>>(q, sh, n, K, gs, static_cast<__half*>(w));
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(MOEB200_ERR_CUDA, "dense_int8_dequant: %s", cudaGetErrorString(e));
  return MOEB200_OK;
}

}  // extern "C"
