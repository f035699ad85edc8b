// Shared device helpers for the moeb200 kernels (sm_100a only).
//
// Everything here is written for Blackwell B200: 1-D bulk TMA copies (cp.async.bulk) completed on
// shared-memory mbarriers, warp-level tensor-core fragments (mma.sync m16n8k16) used as the
// multiply-accumulate engine of the weight-streaming GEMVs, and register-level int4/int8 dequant.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/moeb200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "moeb200 kernels target sm_100a only"
#endif

namespace moeb200 {

// Device-side status word: kernels that wait on anything record why they gave up here instead of
// hanging; the host reads it back through moeb200_check_workspace (moeb200_noalloc_check_status for
// the static scratch of the workspace-free entry point).
enum DevStatus : int32_t {
  kDevOk = 0,
  kDevTimeout = 1,       // an mbarrier wait ran past its iteration budget
  kDevBadIndex = 2,      // an expert / token index outside its range reached a kernel
  kDevMissingExpert = 3  // (informational) a routed expert had no resident record
};

// Iteration budget of every spin-wait. A healthy wait ends within microseconds; 2^22 polls of a
// try_wait (each may suspend for a hardware-chosen interval) is well under a few seconds, after
// which the kernel records kDevTimeout and stops waiting.
constexpr uint32_t kSpinLimit = 1u << 22;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------------------------
// Programmatic dependent launch of the layer's kernel chain (router -> dispatch -> gate/up -> down
// -> finalize). Each kernel is launched with programmatic stream serialization, so its CTAs may be
// scheduled while the previous kernel on the stream drains; every CTA calls chain_wait() before it
// touches global memory, which returns once the previous kernel has completed and its writes are
// visible (immediately for a kernel launched without the attribute). Because every CTA waits, a
// kernel completes only after its predecessor did, so ordering stays transitive along the stream.
// chain_release() lets the next kernel be scheduled early; it does not publish any data.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void chain_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void chain_release() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launches kern<<<grid, block, smem, s>>>(args...) with programmatic stream serialization.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_chained(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                  Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// ---------------------------------------------------------------------------------------------
// mbarrier + 1-D bulk TMA
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Returns true when the phase with the given parity has completed.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: false (and the status word set) if the budget ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int32_t* status) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  if (status) atomicExch(status, kDevTimeout);
  return false;
}

// Global -> shared bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned),
// completing `bytes` transactions on `bar`.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------------------------
// Tensor-core fragment MMA: D(16x8, f32) += A(16x16) * B(16x8), A row-major, B column-major.
// ---------------------------------------------------------------------------------------------
template <typename T>
struct MmaOp;

template <>
struct MmaOp<__half> {
  // c += a * b
  static __device__ __forceinline__ void run(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  // c = a * b (accumulators start from zero registers, no separate clearing)
  static __device__ __forceinline__ void first(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};\n"
        : "=f"(c[0]), "=f"(c[1]), "=f"(c[2]), "=f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
  }
};

template <>
struct MmaOp<__nv_bfloat16> {
  static __device__ __forceinline__ void run(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ void first(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};\n"
        : "=f"(c[0]), "=f"(c[1]), "=f"(c[2]), "=f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
  }
};

// ---------------------------------------------------------------------------------------------
// Register dequantisation to packed 16-bit pairs.
//
// int4 (fp16): in a 32-bit word holding 8 nibbles n0..n7 (nibble i at bits 4i..4i+3, low nibble of
// each byte = even column), masking with 0x000F000F / 0x00F000F0 and OR-ing the fp16 exponent of
// 1024 (0x6400) yields the exact fp16 pairs (1024+n0, 1024+n4) and (1024+16*n1, 1024+16*n5); the
// word shifted by 8 gives (n2, n6) and (n3, n7) the same way. One fused multiply-add per pair then
// removes the offsets exactly: (1024+n) - 1032 = n-8, (1024+16n)/16 - 72 = n-8.
// The column pairs are therefore (c, c+4), (c+1, c+5), (c+2, c+6), (c+3, c+7); the activation
// operand is permuted the same way, so each dot product is unchanged.
// int4 (bf16): same with the bf16 exponent of 128 (0x4300): (128+n) - 136, (128+16n)/16 - 16.
// ---------------------------------------------------------------------------------------------
template <typename T>
struct Dq;

template <>
struct Dq<__half> {
  static __device__ __forceinline__ void int4x8(uint32_t w, uint32_t& p04, uint32_t& p15, uint32_t& p26,
                                                uint32_t& p37) {
    const uint32_t w8 = w >> 8;
    uint32_t a, b, c, d;
    asm("lop3.b32 %0, %1, 0x000F000F, 0x64006400, 0xEA;" : "=r"(a) : "r"(w));
    asm("lop3.b32 %0, %1, 0x00F000F0, 0x64006400, 0xEA;" : "=r"(b) : "r"(w));
    asm("lop3.b32 %0, %1, 0x000F000F, 0x64006400, 0xEA;" : "=r"(c) : "r"(w8));
    asm("lop3.b32 %0, %1, 0x00F000F0, 0x64006400, 0xEA;" : "=r"(d) : "r"(w8));
    const uint32_t k1032 = 0x64086408u;  // (1032, 1032)
    const uint32_t k16 = 0x2C002C00u;    // (1/16, 1/16)
    const uint32_t km72 = 0xD480D480u;   // (-72, -72)
    asm("sub.f16x2 %0, %1, %2;" : "=r"(p04) : "r"(a), "r"(k1032));
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(p15) : "r"(b), "r"(k16), "r"(km72));
    asm("sub.f16x2 %0, %1, %2;" : "=r"(p26) : "r"(c), "r"(k1032));
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(p37) : "r"(d), "r"(k16), "r"(km72));
  }
  // int8: word = 4 signed bytes at columns c..c+3 -> (c, c+1), (c+2, c+3).
  static __device__ __forceinline__ void int8x4(uint32_t w, uint32_t& p01, uint32_t& p23) {
    const uint32_t u = w ^ 0x80808080u;  // signed -> biased +128
    uint32_t a, b;
    asm("prmt.b32 %0, %1, %2, 0x4140;" : "=r"(a) : "r"(u), "r"(0x64646464u));
    asm("prmt.b32 %0, %1, %2, 0x4342;" : "=r"(b) : "r"(u), "r"(0x64646464u));
    const uint32_t k1152 = 0x64806480u;  // (1152, 1152) = 1024 + 128
    asm("sub.f16x2 %0, %1, %2;" : "=r"(p01) : "r"(a), "r"(k1152));
    asm("sub.f16x2 %0, %1, %2;" : "=r"(p23) : "r"(b), "r"(k1152));
  }
  static __device__ __forceinline__ uint32_t pack_f32(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

template <>
struct Dq<__nv_bfloat16> {
  static __device__ __forceinline__ void int4x8(uint32_t w, uint32_t& p04, uint32_t& p15, uint32_t& p26,
                                                uint32_t& p37) {
    // bf16 keeps only 7 mantissa bits, so every nibble is first shifted down to bits 0..3 (a nibble
    // at bits 4..7 would reach the exponent): (128 + n) - 136 = n - 8, exact.
    uint32_t a, b, c, d;
    asm("lop3.b32 %0, %1, 0x000F000F, 0x43004300, 0xEA;" : "=r"(a) : "r"(w));
    asm("lop3.b32 %0, %1, 0x000F000F, 0x43004300, 0xEA;" : "=r"(b) : "r"(w >> 4));
    asm("lop3.b32 %0, %1, 0x000F000F, 0x43004300, 0xEA;" : "=r"(c) : "r"(w >> 8));
    asm("lop3.b32 %0, %1, 0x000F000F, 0x43004300, 0xEA;" : "=r"(d) : "r"(w >> 12));
    const uint32_t one = 0x3F803F80u;    // (1, 1)
    const uint32_t km136 = 0xC308C308u;  // (-136, -136)
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(p04) : "r"(a), "r"(one), "r"(km136));
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(p15) : "r"(b), "r"(one), "r"(km136));
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(p26) : "r"(c), "r"(one), "r"(km136));
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(p37) : "r"(d), "r"(one), "r"(km136));
  }
  // int8 -> bf16: bf16 cannot hold 0..255 at unit spacing under one exponent, so each byte goes
  // through an exact fp32 (2^23 + u) - (2^23 + 128) and the pair is packed (exact: |b| <= 128).
  static __device__ __forceinline__ void int8x4(uint32_t w, uint32_t& p01, uint32_t& p23) {
    const uint32_t u = w ^ 0x80808080u;
    uint32_t f0, f1, f2, f3;
    asm("prmt.b32 %0, %1, %2, 0x7540;" : "=r"(f0) : "r"(u), "r"(0x4B000000u));
    asm("prmt.b32 %0, %1, %2, 0x7541;" : "=r"(f1) : "r"(u), "r"(0x4B000000u));
    asm("prmt.b32 %0, %1, %2, 0x7542;" : "=r"(f2) : "r"(u), "r"(0x4B000000u));
    asm("prmt.b32 %0, %1, %2, 0x7543;" : "=r"(f3) : "r"(u), "r"(0x4B000000u));
    const float off = 8388736.0f;  // 2^23 + 128
    p01 = pack_f32(__uint_as_float(f0) - off, __uint_as_float(f1) - off);
    p23 = pack_f32(__uint_as_float(f2) - off, __uint_as_float(f3) - off);
  }
  static __device__ __forceinline__ uint32_t pack_f32(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_f32<float>(float v) {
  return v;
}

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) {
  return __float2half_rn(v);
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ float from_f32<float>(float v) {
  return v;
}

// 16-bit pair (lo, hi) from two 16-bit values held in the low halves of two registers.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

__device__ __forceinline__ void red_add_f32(float* p, float v) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

}  // namespace moeb200
