// Fused decode kernel: the whole expert half of an MoE layer in ONE persistent launch --
// gate/up GEMV + SwiGLU, down GEMV, weighted combine and the cast to the activation type.
//
// Replaces, for decode batches (work items of at most 8 tokens), the two-launch grouped GEMV of
// gemv.cu and its finalize kernel. The computation is moelab's grouped expert product
// (kernels.py `_grp4_up`/`_grp4_down` 312-396, `_grp8_*` 667-740, `_grpf_*` 398-451; the combine
// of runtime.py:342-353):
//
//   h[j, r]    = silu(gate_r . x_tok(j)) * (up_r . x_tok(j))        every pair j of an item
//   out[t, r]  = sum over the pairs j of token t of  w_j * (down_r . h[j])
//
// Work units. An item (<= 8 pairs of one (expert, precision)) has I/8 gate/up units (8 gate rows
// and the matching 8 up rows: one 16-row tensor-core tile whose rows 0..7 are gate and 8..15 up,
// so SwiGLU pairs sit in one lane) and H/16 down units (16 rows), numbered item by item (items
// slot-major, as dispatch numbers them). Each phase is split statically: every CTA takes the
// contiguous run of units whose bytes make up its 1/G share (a CTA's work then touches one or two
// items per phase, so the per-item latencies -- activation rows, h readiness -- are paid rarely).
// A job is 1, 2 or 4 consecutive units (tiles) of one item and phase. The producer moves a job's
// weight rows with one TMA tensor load per tile (one 3-D tensor map per precision and phase, based
// below every resident
// record, so a record's rows are reached through the row coordinate and no map is built per
// record), landing in shared memory with the 128-byte swizzle: the consumers' row-parallel reads
// are then free of bank conflicts. Scales and activation rows come with 1-D bulk copies.
//
// Pipeline. One CTA per SM: a producer lane, kDecCons consumer warps and one epilogue warp. The
// producer and the consumers share a byte ring of shared memory and kDecSlots job slots (descriptor
// + full/empty mbarriers); the producer runs ahead by as many jobs as the ring holds. When a job
// starts a new (item, phase), it also copies the item's activation rows (x rows for gate/up; for
// down the item's h rows, once every gate/up unit of the item has finished -- a per-item counter,
// waited on with a bounded spin).
//
// Consumers. Every job is computed by all consumer warps, each owning a fixed slice of K (64-column
// groups); a warp keeps its slice of the item's activations as mma.sync B fragments in registers
// for as long as the item lasts, so a job costs per weight only the shared-memory load, the
// dequantisation and the MMA. Integer records are dequantised without removing their offset:
//   int4, fp16 activations: 1024 + q (even nibbles) and 1024 + 16 q (odd nibbles, whose activation
//     operand is pre-divided by 16), i.e. 5 instructions per 8 weights;
//   int4, bf16 activations: 128 + q;  int8, fp16 activations: 1152 + q;
// the products are exact and each 64-column group's fp32 partial gets the offset removed as
// (partial - c * sum of the group's activations) before it is multiplied by the group's fp16 scale.
// (int8 with bf16 activations converts exactly through fp32; float records are used as stored.)
//
// Epilogue. Each consumer stores its partial sums of a job into its own slice of one of kDecRed
// shared-memory buffers; the epilogue warp adds the slices in warp order (deterministic, no shared
// atomics) and does all global work, taking the jobs in order, so no
// consumer ever waits on global memory: SwiGLU into h (gate/up), whose items' counters it raises in
// batches behind one fence per batch, or w_j-weighted fp32 reductions into acc (down). When a CTA
// has no job left it counts itself done; once every CTA is done, each casts its slice of acc into
// `out`, so no finalize launch follows.
#include <algorithm>
#include <type_traits>

#include "gemv.cuh"
#include "tma.cuh"

namespace moeb200 {

namespace {

constexpr int kDecCons = 8;                       // consumer warps (0 .. kDecCons-1)
constexpr int kDecProd = kDecCons;                // producer warp
constexpr int kDecEpi = kDecCons + 1;             // epilogue warp
constexpr int kDecThreads = 32 * (kDecCons + 2);
constexpr int kDecSlots = 16;                     // job slots
constexpr int kDecRed = 2;                        // reduction buffers
constexpr int kDecMT = 4;                         // 16-row tiles per job at most
constexpr uint32_t kDecJobW = 64 * 1024;          // weight bytes per job at most (or one unit)
constexpr int kDecCmax = 4;                       // 64-column groups of a consumer's K slice at most
constexpr int kDecRing = 188 * 1024;              // bytes of the job ring

struct alignas(16) DecJob {
  int32_t item;        // -1: no more jobs
  int32_t up;          // 1: gate/up, 0: down
  int32_t rb0;         // first unit of the job (gate/up: 8 gate rows; down: 16 rows)
  int32_t n;           // units (16-row tiles)
  int32_t start;       // the item's first sorted pair (h row)
  int32_t ntok;        // the item's pairs
  int32_t slot;        // precision slot
  int32_t fresh;       // the job starts a new (item, phase): its activation rows follow at xo
  uint32_t w0, w1;     // ring offsets of the weight rows (gate/up: gate rows, then up rows)
  uint32_t s0, s1;     // ring offsets of the scale rows
  uint32_t xo;         // ring offset of the activation rows (fresh jobs)
  int32_t _pad[3];
};
static_assert(sizeof(DecJob) == 64, "DecJob layout");

// Tensor maps of the weight fields, per precision slot and phase (0 gate/up, 1 down): uint8
// [segment][row][128] views of all memory from tma_base on, rows of the field's row pitch, boxes of
// one tile (8 rows for gate/up, 16 for down) x every 128-byte segment of a row, 128-byte swizzle.
struct alignas(64) DecMaps {
  CUtensorMap m[4][2];
};

__device__ __forceinline__ void tma3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// Byte offset, inside a tile's box of R rows, of byte b of row r (rows of whole 128-byte segments,
// laid out segment-major; 16-byte units XOR-swizzled by row % 8 as TMA writes them).
__device__ __forceinline__ uint32_t swz_off(int R, int r, int b) {
  return (uint32_t)((((b >> 7) * R + r) << 7) + ((((b >> 4) & 7) ^ (r & 7)) << 4) + (b & 15));
}

// What the epilogue warp needs of a job, written beside its reduction buffer by the consumers.
struct alignas(16) RedHdr {
  int32_t item;  // -1: no more jobs
  int32_t up;
  int32_t rb0;
  int32_t n;
  int32_t start;
  int32_t ntok;
  int32_t _pad[2];
};

// Shared-memory map (after the 1024-byte aligned base).
constexpr int kRedSlice = kDecMT * 4 * 32;                        // one warp's partials [kDecMT][4][32]
constexpr int kRedFloats = kDecCons * kRedSlice;                  // one reduction buffer: a slice per warp
constexpr int kOffJobs = kDecRing;
constexpr int kOffBars = kOffJobs + kDecSlots * (int)sizeof(DecJob);
constexpr int kOffVend = kOffBars + 2 * kDecSlots * 8;
constexpr int kOffRed = kOffVend + kDecSlots * 4;                 // [kDecRed] buffers, fp32
constexpr int kOffHdr = kOffRed + kDecRed * kRedFloats * 4;       // [kDecRed] RedHdr
constexpr int kOffRbar = kOffHdr + kDecRed * (int)sizeof(RedHdr);  // sums_ready[kDecRed], buf_free[kDecRed]
constexpr int kDecSmem = kOffRbar + 16 * kDecRed + 1024;           // + alignment slack
static_assert(kDecSmem <= 227 * 1024, "decode kernel shared memory");

enum DecKind : int { kKI4 = 0, kKI8 = 1, kKF = 2 };

__device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__device__ __forceinline__ int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_complete_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.complete_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive1(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ uint64_t gtime() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ int32_t ld_acquire(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Bounded spin until *p >= target (acquire); false (status set) if the budget ran out.
__device__ __forceinline__ bool wait_counter(const int32_t* p, int32_t target, int32_t* status) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (ld_acquire(p) >= target) return true;
    __nanosleep(256);
  }
  if (status) atomicExch(status, kDevTimeout);
  return false;
}

// ---- dequantisation with the offset kept (the group correction removes it) -----------------------
template <typename AT>
struct Dec;

template <>
struct Dec<__half> {
  // 8 nibbles -> (1024+n0, 1024+n4), (1024+16n1, 1024+16n5) [lo]; (1024+n2, 1024+n6), (1024+16n3,
  // 1024+16n7) [hi]
  static __device__ __forceinline__ void i4_lo(uint32_t w, uint32_t& p04, uint32_t& p15) {
    asm("lop3.b32 %0, %1, 0x000F000F, 0x64006400, 0xEA;" : "=r"(p04) : "r"(w));
    asm("lop3.b32 %0, %1, 0x00F000F0, 0x64006400, 0xEA;" : "=r"(p15) : "r"(w));
  }
  static __device__ __forceinline__ void i4_hi(uint32_t w, uint32_t& p26, uint32_t& p37) { i4_lo(w >> 8, p26, p37); }
  // 4 signed bytes -> (1152+q0, 1152+q1), (1152+q2, 1152+q3)
  static __device__ __forceinline__ void i8(uint32_t w, uint32_t& p01, uint32_t& p23) {
    const uint32_t u = w ^ 0x80808080u;
    asm("prmt.b32 %0, %1, %2, 0x4140;" : "=r"(p01) : "r"(u), "r"(0x64646464u));
    asm("prmt.b32 %0, %1, %2, 0x4342;" : "=r"(p23) : "r"(u), "r"(0x64646464u));
  }
  static constexpr float kEven4 = 1032.f;  // correction per activation, even nibbles
  static constexpr float kOdd4 = 1152.f;   // per (activation / 16), odd nibbles: (1024 + 16q) x/16 - (q-8) x
  static constexpr float kI8 = 1152.f;
  static constexpr bool kScaleOdd = true;  // odd-nibble activations are divided by 16
};

template <>
struct Dec<__nv_bfloat16> {
  // bf16 keeps 7 mantissa bits: every nibble is shifted to bits 0..3 first -> 128 + n
  static __device__ __forceinline__ void i4_lo(uint32_t w, uint32_t& p04, uint32_t& p15) {
    asm("lop3.b32 %0, %1, 0x000F000F, 0x43004300, 0xEA;" : "=r"(p04) : "r"(w));
    asm("lop3.b32 %0, %1, 0x000F000F, 0x43004300, 0xEA;" : "=r"(p15) : "r"(w >> 4));
  }
  static __device__ __forceinline__ void i4_hi(uint32_t w, uint32_t& p26, uint32_t& p37) { i4_lo(w >> 8, p26, p37); }
  // exact values q (through fp32), no offset
  static __device__ __forceinline__ void i8(uint32_t w, uint32_t& p01, uint32_t& p23) { Dq<__nv_bfloat16>::int8x4(w, p01, p23); }
  static constexpr float kEven4 = 136.f;
  static constexpr float kOdd4 = 136.f;
  static constexpr float kI8 = 0.f;
  static constexpr bool kScaleOdd = false;
};

// ---- one tile over the warp's K slice ----------------------------------------------------------------
// rg / rh: shared address of the tile's rows g and g+8 inside its swizzled box (row base); colo[cl]:
// offset of the lane's bytes of the warp's cl-th group from a row base (every row the lane reads has
// r % 8 == g); sg / sh: the two rows' scale rows. B[cl]: the activation operand of group cl (8
// registers), corr[cl]: the group's offset correction for the lane's two accumulator tokens.
// tot = the tile's partial for rows (g, g+8) x tokens (2t, 2t+1). The body covers up to NC groups
// (nc of them live), whose MMA chains are independent and advance in lockstep, one MMA each in turn,
// so the MMA latency is hidden; the tile loop around it stays a runtime loop (the code stays small
// enough for the instruction cache).
template <typename AT, int NC>
__device__ __forceinline__ void tile_i4(const uint8_t* rg, const uint8_t* rh, const uint8_t* sg, const uint8_t* sh,
                                        int c0, int nc, const uint32_t (&colo)[kDecCmax],
                                        const uint32_t (&B)[kDecCmax][8], const float (&corr)[kDecCmax][2],
                                        float (&tot)[4]) {
  uint2 wa[NC], wb[NC];
  float s0[NC], s1[NC], d[NC][4];
#pragma unroll
  for (int cl = 0; cl < NC; ++cl)
    if (cl < nc) {
      wa[cl] = *reinterpret_cast<const uint2*>(rg + colo[cl]);
      wb[cl] = *reinterpret_cast<const uint2*>(rh + colo[cl]);
      s0[cl] = __half2float(reinterpret_cast<const __half*>(sg)[c0 + cl]);
      s1[cl] = __half2float(reinterpret_cast<const __half*>(sh)[c0 + cl]);
    }
#pragma unroll
  for (int h = 0; h < 4; ++h) {  // word j = h / 2 of the lane's two (8 columns each); its lo then hi pairs
    const int j = h >> 1;
    uint32_t a[NC][4];
#pragma unroll
    for (int cl = 0; cl < NC; ++cl)
      if (cl < nc) {
        const uint32_t x = j ? wa[cl].y : wa[cl].x, y = j ? wb[cl].y : wb[cl].x;
        if (h & 1) {
          Dec<AT>::i4_hi(x, a[cl][0], a[cl][2]);
          Dec<AT>::i4_hi(y, a[cl][1], a[cl][3]);
        } else {
          Dec<AT>::i4_lo(x, a[cl][0], a[cl][2]);
          Dec<AT>::i4_lo(y, a[cl][1], a[cl][3]);
        }
      }
#pragma unroll
    for (int cl = 0; cl < NC; ++cl)
      if (cl < nc) {
        if (h == 0)
          MmaOp<AT>::first(d[cl], a[cl], B[cl][0], B[cl][1]);
        else
          MmaOp<AT>::run(d[cl], a[cl], B[cl][2 * h], B[cl][2 * h + 1]);
      }
  }
#pragma unroll
  for (int cl = 0; cl < NC; ++cl)
    if (cl < nc) {
      tot[0] = fmaf(s0[cl], d[cl][0] - corr[cl][0], tot[0]);
      tot[1] = fmaf(s0[cl], d[cl][1] - corr[cl][1], tot[1]);
      tot[2] = fmaf(s1[cl], d[cl][2] - corr[cl][0], tot[2]);
      tot[3] = fmaf(s1[cl], d[cl][3] - corr[cl][1], tot[3]);
    }
}

template <typename AT, int NC>
__device__ __forceinline__ void tile_i8(const uint8_t* rg, const uint8_t* rh, const uint8_t* sg, const uint8_t* sh,
                                        int c0, int nc, const uint32_t (&colo)[kDecCmax],
                                        const uint32_t (&B)[kDecCmax][8], const float (&corr)[kDecCmax][2],
                                        float (&tot)[4]) {
  uint4 wa[NC], wb[NC];
  float s0[NC], s1[NC], d[NC][4];
#pragma unroll
  for (int cl = 0; cl < NC; ++cl)
    if (cl < nc) {
      wa[cl] = *reinterpret_cast<const uint4*>(rg + colo[cl]);
      wb[cl] = *reinterpret_cast<const uint4*>(rh + colo[cl]);
      s0[cl] = __half2float(reinterpret_cast<const __half*>(sg)[c0 + cl]);
      s1[cl] = __half2float(reinterpret_cast<const __half*>(sh)[c0 + cl]);
    }
#pragma unroll
  for (int j = 0; j < 4; ++j) {  // the lane's four words (4 columns each) of a group
#pragma unroll
    for (int cl = 0; cl < NC; ++cl)
      if (cl < nc) {
        const uint32_t x = j == 0 ? wa[cl].x : j == 1 ? wa[cl].y : j == 2 ? wa[cl].z : wa[cl].w;
        const uint32_t y = j == 0 ? wb[cl].x : j == 1 ? wb[cl].y : j == 2 ? wb[cl].z : wb[cl].w;
        uint32_t A[4];
        Dec<AT>::i8(x, A[0], A[2]);
        Dec<AT>::i8(y, A[1], A[3]);
        if (j == 0)
          MmaOp<AT>::first(d[cl], A, B[cl][0], B[cl][1]);
        else
          MmaOp<AT>::run(d[cl], A, B[cl][2 * j], B[cl][2 * j + 1]);
      }
  }
#pragma unroll
  for (int cl = 0; cl < NC; ++cl)
    if (cl < nc) {
      tot[0] = fmaf(s0[cl], d[cl][0] - corr[cl][0], tot[0]);
      tot[1] = fmaf(s0[cl], d[cl][1] - corr[cl][1], tot[1]);
      tot[2] = fmaf(s1[cl], d[cl][2] - corr[cl][0], tot[2]);
      tot[3] = fmaf(s1[cl], d[cl][3] - corr[cl][1], tot[3]);
    }
}

// float records of the activation type: used as stored. colo[cl] points at the lane's first 16
// bytes of the group (an even 16-byte unit; the second is the next unit, bit 0 of the unit flipped).
template <typename AT, int NC>
__device__ __forceinline__ void tile_f(const uint8_t* rg, const uint8_t* rh, int nc, const uint32_t (&colo)[kDecCmax],
                                       const uint32_t (&B)[kDecCmax][8], float (&tot)[4]) {
  float d[NC][4];
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    uint4 fa[NC], fb[NC];
#pragma unroll
    for (int cl = 0; cl < NC; ++cl)
      if (cl < nc) {
        fa[cl] = *reinterpret_cast<const uint4*>(rg + (colo[cl] ^ (q << 4)));
        fb[cl] = *reinterpret_cast<const uint4*>(rh + (colo[cl] ^ (q << 4)));
      }
#pragma unroll
    for (int cl = 0; cl < NC; ++cl)
      if (cl < nc) {
        const uint32_t A0[4] = {fa[cl].x, fb[cl].x, fa[cl].y, fb[cl].y};
        if (q == 0)
          MmaOp<AT>::first(d[cl], A0, B[cl][0], B[cl][1]);
        else
          MmaOp<AT>::run(d[cl], A0, B[cl][4], B[cl][5]);
      }
#pragma unroll
    for (int cl = 0; cl < NC; ++cl)
      if (cl < nc) {
        const uint32_t A1[4] = {fa[cl].z, fb[cl].z, fa[cl].w, fb[cl].w};
        MmaOp<AT>::run(d[cl], A1, B[cl][2 + 4 * q], B[cl][3 + 4 * q]);
      }
  }
#pragma unroll
  for (int cl = 0; cl < NC; ++cl)
    if (cl < nc)
#pragma unroll
      for (int e = 0; e < 4; ++e) tot[e] += d[cl][e];
}

__device__ __forceinline__ float2 pair_f32_h(uint32_t v) {
  const __half2 h = *reinterpret_cast<const __half2*>(&v);
  return __half22float2(h);
}
__device__ __forceinline__ float2 pair_f32_b(uint32_t v) {
  const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&v);
  return __bfloat1622float2(h);
}
template <typename AT>
__device__ __forceinline__ float pair_sum(uint32_t v) {
  float2 f;
  if constexpr (std::is_same<AT, __half>::value)
    f = pair_f32_h(v);
  else
    f = pair_f32_b(v);
  return f.x + f.y;
}

// The warp's activation operand for a new item: lane (g, t) holds token g's 16 columns
// [64c + 16t, +16) of each of its groups c (zeros for g >= ntok), arranged for the item's record kind,
// and the per-group offset corrections of the lane's accumulator tokens 2t and 2t+1.
template <typename AT>
__device__ __forceinline__ void load_operand(const uint8_t* xrow, bool on, int kind, int c0, int nc, int g, int t,
                                             uint32_t (&B)[kDecCmax][8], float (&corr)[kDecCmax][2]) {
#pragma unroll
  for (int cl = 0; cl < kDecCmax; ++cl) {
    uint32_t v[8];
    if (on && cl < nc) {
      const uint4 a = *reinterpret_cast<const uint4*>(xrow + (c0 + cl) * 128 + t * 32);
      const uint4 b = *reinterpret_cast<const uint4*>(xrow + (c0 + cl) * 128 + t * 32 + 16);
      v[0] = a.x;
      v[1] = a.y;
      v[2] = a.z;
      v[3] = a.w;
      v[4] = b.x;
      v[5] = b.y;
      v[6] = b.z;
      v[7] = b.w;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0u;
    }
    float c = 0.f;
    if (kind == kKI4) {
      // columns (x0, x4), (x1, x5), (x2, x6), (x3, x7) of each 8-column word, as the nibble pairs
      float se = 0.f, so = 0.f;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        uint32_t p04 = prmt(v[4 * j], v[4 * j + 2], 0x5410), p15 = prmt(v[4 * j], v[4 * j + 2], 0x7632);
        uint32_t p26 = prmt(v[4 * j + 1], v[4 * j + 3], 0x5410), p37 = prmt(v[4 * j + 1], v[4 * j + 3], 0x7632);
        if constexpr (Dec<AT>::kScaleOdd) {
          const __half2 k16 = __float2half2_rn(0.0625f);
          __half2 h15 = __hmul2(*reinterpret_cast<__half2*>(&p15), k16);
          __half2 h37 = __hmul2(*reinterpret_cast<__half2*>(&p37), k16);
          p15 = *reinterpret_cast<uint32_t*>(&h15);
          p37 = *reinterpret_cast<uint32_t*>(&h37);
        }
        B[cl][4 * j] = p04;
        B[cl][4 * j + 1] = p15;
        B[cl][4 * j + 2] = p26;
        B[cl][4 * j + 3] = p37;
        se += pair_sum<AT>(p04) + pair_sum<AT>(p26);
        so += pair_sum<AT>(p15) + pair_sum<AT>(p37);
      }
      c = Dec<AT>::kEven4 * se + Dec<AT>::kOdd4 * so;
    } else {
      float sa = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        B[cl][i] = v[i];
        sa += pair_sum<AT>(v[i]);
      }
      c = kind == kKI8 ? Dec<AT>::kI8 * sa : 0.f;
    }
    // token g's correction = sum over the 4 lanes of row g; the accumulators of lane (g, t) hold
    // tokens 2t and 2t+1, whose sums sit in lanes 8t and 8t+4
    c += __shfl_xor_sync(0xffffffffu, c, 1);
    c += __shfl_xor_sync(0xffffffffu, c, 2);
    corr[cl][0] = __shfl_sync(0xffffffffu, c, 8 * t);
    corr[cl][1] = __shfl_sync(0xffffffffu, c, 8 * t + 4);
  }
}

// One job of n tiles for one consumer warp: once the job's reduction buffer is free (use seq /
// kDecRed of it), each tile's partial sums over the warp's K slice go into the warp's slice rb of the
// buffer; then the ring slot is released. false if a bounded wait gave up.
template <typename AT>
__device__ __forceinline__ bool consume(int kind, int n, const uint8_t* rg0, const uint8_t* rh0, uint32_t tile,
                                     const uint8_t* sg0, const uint8_t* sh0, uint32_t sstep, int c0, int nc,
                                     const uint32_t (&colo)[kDecCmax], const uint32_t (&B)[kDecCmax][8],
                                     const float (&corr)[kDecCmax][2], int lane, uint64_t* empty_s, uint64_t* free_b,
                                     uint32_t seq, float* rb, int32_t* status) {
  int ok = 1;
  if (lane == 0 && seq >= kDecRed) ok = mbar_wait(free_b, ((seq / kDecRed) - 1) & 1, status);
  if (!__shfl_sync(0xffffffffu, ok, 0)) return false;
  for (int m = 0; m < n; ++m) {
    const uint8_t* rg = rg0 + m * tile;
    const uint8_t* rh = rh0 + m * tile;
    const uint8_t* sg = sg0 + m * sstep;
    const uint8_t* sh = sh0 + m * sstep;
    float tot[4] = {0.f, 0.f, 0.f, 0.f};
    if (kind == kKI4) {
      if (nc <= 2)
        tile_i4<AT, 2>(rg, rh, sg, sh, c0, nc, colo, B, corr, tot);
      else
        tile_i4<AT, 4>(rg, rh, sg, sh, c0, nc, colo, B, corr, tot);
    } else if (kind == kKI8) {
      if (nc <= 2)
        tile_i8<AT, 2>(rg, rh, sg, sh, c0, nc, colo, B, corr, tot);
      else
        tile_i8<AT, 4>(rg, rh, sg, sh, c0, nc, colo, B, corr, tot);
    } else {
      if (nc <= 2)
        tile_f<AT, 2>(rg, rh, nc, colo, B, tot);
      else
        tile_f<AT, 4>(rg, rh, nc, colo, B, tot);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) rb[(m * 4 + i) * 32 + lane] = tot[i];
  }
  __syncwarp();
  if (lane == 0) mbar_arrive1(empty_s);  // the job's ring bytes are no longer read by this warp
  return true;
}

template <typename AT>
__global__ void __launch_bounds__(kDecThreads, 1) decode_kernel(const DecodeParams p, const __grid_constant__ DecMaps tm) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  uint8_t* ring = smem;
  DecJob* jobs = reinterpret_cast<DecJob*>(smem + kOffJobs);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBars);
  uint64_t* empty = full + kDecSlots;
  uint32_t* vend = reinterpret_cast<uint32_t*>(smem + kOffVend);
  float* red = reinterpret_cast<float*>(smem + kOffRed);
  RedHdr* hdr = reinterpret_cast<RedHdr*>(smem + kOffHdr);
  // reduction buffer b: sums_ready[b] completes when every consumer has added its partials of the
  // buffer's current job; buf_free[b] when the epilogue warp has taken them (use k of a buffer
  // waits for release k-1)
  uint64_t* sums_ready = reinterpret_cast<uint64_t*>(smem + kOffRbar);
  uint64_t* buf_free = sums_ready + kDecRed;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kDecSlots; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kDecCons);
    }
    for (int b = 0; b < kDecRed; ++b) {
      mbar_init(&sums_ready[b], kDecCons);
      mbar_init(&buf_free[b], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();
  chain_wait();
  chain_release();
  const int n_items = *p.n_items;

  if (warp == kDecProd) {
    // ======================= producer (one lane) =======================
    if (lane != 0) return;
    const int G = gridDim.x;
    const int Uup = p.I / 8, Udn = p.H / 16;
    const int64_t nup = (int64_t)n_items * Uup;
    // Static byte-balanced partition of each phase: units are numbered item by item, items slot-major,
    // so a phase's cumulative bytes are piecewise linear over the precision slots; this CTA takes the
    // units whose middle byte falls in its 1/G share (every CTA computes the same split).
    int sbeg[5];
#pragma unroll
    for (int i = 0; i < 5; ++i) sbeg[i] = i <= p.nprec ? p.slot_items[i] : n_items;
    auto unit_bytes = [&](int sl, bool upp) -> int64_t {
      const LayoutDev L = p.lay[sl];
      const bool ii = L.wtype == MOEB200_I4 || L.wtype == MOEB200_I8;
      const int K = upp ? p.H : p.I;
      return 16ll * K * gemv_wbits(L.wtype) / 8 + (ii ? 16ll * (K / 64) * 2 : 0);
    };
    // units of the phase whose middle byte lies below byte x
    auto units_below = [&](bool upp, int64_t x) -> int64_t {
      const int U = upp ? Uup : Udn;
      int64_t ub = 0, bb = 0;
      for (int sl = 0; sl < p.nprec; ++sl) {
        const int64_t nu = (int64_t)(sbeg[sl + 1] - sbeg[sl]) * U, w = unit_bytes(sl, upp);
        if (x < bb + nu * w) return ub + min64(nu, max64(0, (x - bb + w / 2) / w));
        ub += nu;
        bb += nu * w;
      }
      return ub;
    };
    auto phase_bytes = [&](bool upp) -> int64_t {
      const int U = upp ? Uup : Udn;
      int64_t bb = 0;
      for (int sl = 0; sl < p.nprec; ++sl) bb += (int64_t)(sbeg[sl + 1] - sbeg[sl]) * U * unit_bytes(sl, upp);
      return bb;
    };
    const int64_t Bu = phase_bytes(true), Bd = phase_bytes(false);
    // this CTA's units: [cur, cend) of gate/up, then [dcur, dend) of down (offset by nup)
    int64_t cur = units_below(true, Bu * blockIdx.x / G), cend = units_below(true, Bu * (blockIdx.x + 1) / G);
    const int64_t dcur = nup + units_below(false, Bd * blockIdx.x / G);
    const int64_t dend = nup + units_below(false, Bd * (blockIdx.x + 1) / G);
    bool in_down = false;
    uint32_t seq = 0, oldest = 0, vhead = 0, vtail = 0;
    int cur_item = -1, cur_up = -1;
    Item it{};
    bool ok = true;
    // Frees the oldest jobs (in issue order, as the consumers release them) until need_ring bytes
    // fit after vhead and a job slot is free. With no job in flight the whole ring is free, including
    // a lap tail skipped by a wrap (which vtail alone would still count as in use).
    auto free_until = [&](uint32_t need_ring) -> bool {
      while (true) {
        if (oldest == seq) vtail = vhead;
        const bool ring_full = need_ring && vhead + need_ring - vtail > (uint32_t)kDecRing;
        if (!ring_full && oldest + kDecSlots > seq) return true;
        const uint32_t os = oldest % kDecSlots;
        if (!mbar_wait(&empty[os], (oldest / kDecSlots) & 1, p.status)) return false;
        vtail = vend[os];
        ++oldest;
      }
    };
    while (true) {
      if (cur >= cend) {
        if (in_down || dcur >= dend) break;
        in_down = true;
        cur = dcur;
        cend = dend;
      }
      const bool up = cur < nup;
      const int64_t v = up ? cur : cur - nup;
      const int U = up ? Uup : Udn;
      const int item = (int)(v / U), rb0 = (int)(v - (int64_t)item * U);
      if (item < 0 || item >= n_items) {  // a unit past the call's items: a bad partition, never issued
        atomicExch(p.status, kDevBadIndex);
        ok = false;
        break;
      }
      const bool fresh = item != cur_item || (int)up != cur_up;
      if (item != cur_item) it = p.items[item];
      if (it.slot < 0 || it.slot >= p.nprec || it.ntok < 1 || it.ntok > 8) {
        atomicExch(p.status, kDevBadIndex);
        ok = false;
        break;
      }
      cur_item = item;
      cur_up = up;
      const LayoutDev L = p.lay[it.slot];
      const bool isint = L.wtype == MOEB200_I4 || L.wtype == MOEB200_I8;
      const int K = up ? p.H : p.I;
      const uint32_t rowb = (uint32_t)(K * gemv_wbits(L.wtype) / 8);
      const uint32_t unit_w = 16u * rowb;
      const uint32_t srow = isint ? (uint32_t)(K / 64) * 2u : 0u;
      const int nmax = max(1, min(kDecMT, (int)(kDecJobW / unit_w)));
      int n = (int)min64(min64(nmax, cend - cur), U - rb0);
      n = n >= 4 ? 4 : n >= 2 ? 2 : 1;  // jobs of 1, 2 or 4 tiles (the consumers' code is specialised on it)
      const uint32_t wb = n * unit_w, sb = n * 16u * srow;
      const uint32_t xb = fresh ? (uint32_t)it.ntok * K * 2u : 0u;
      // the item's token rows (gate/up), loaded before anything waits
      int tok[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) tok[j] = (up && fresh && j < it.ntok) ? __ldg(p.pos + it.start + j) / p.k : 0;
      // weight boxes start on 1024-byte boundaries (the 128-byte swizzle repeats every 1024 bytes)
      const uint32_t wba = (wb + 1023u) & ~1023u, sba = (sb + 127u) & ~127u;
      const uint32_t need = (wba + sba + xb + 1023u) & ~1023u;
      if (need > (uint32_t)kDecRing) {  // cannot happen for layouts decode_supported accepts
        atomicExch(p.status, kDevBadIndex);
        ok = false;
        break;
      }
      if ((vhead % kDecRing) + need > (uint32_t)kDecRing) vhead += kDecRing - (vhead % kDecRing);
      ok = free_until(need);
      if (!ok) break;
      const uint32_t s = seq % kDecSlots;
      const uint32_t off = vhead % kDecRing;
      vend[s] = vhead + need;
      vhead += need;
      DecJob& d = jobs[s];
      d.item = item;
      d.up = up;
      d.rb0 = rb0;
      d.n = n;
      d.start = it.start;
      d.ntok = it.ntok;
      d.slot = it.slot;
      d.fresh = fresh;
      d.w0 = off;
      d.w1 = off + (up ? wb / 2 : 0u);  // gate tiles, then up tiles (each a multiple of 1024 bytes)
      d.s0 = off + wba;
      d.s1 = off + wba + (up ? sb / 2 : 0u);
      d.xo = off + wba + sba;
      mbar_expect_tx(&full[s], wb + sb + xb);
      const uint8_t* q = reinterpret_cast<const uint8_t*>(up ? it.p_guq : it.p_dnq);
      const uint8_t* sc = reinterpret_cast<const uint8_t*>(up ? it.p_gus : it.p_dns);
      // the field's first row in the maps' row coordinates (records lie on 4096-byte multiples above
      // tma_base, row pitches divide 4096 and the field offsets)
      const int64_t dq = reinterpret_cast<int64_t>(q) - p.tma_base;
      const int64_t row0 = dq / (int64_t)rowb;
      if (dq < 0 || dq % (int64_t)rowb != 0 || row0 + 2 * p.I + p.H > 0x7fffffffll) {
        atomicExch(p.status, kDevBadIndex);  // cannot happen with the runtime's records: skip the rows
        mbar_complete_tx(&full[s], wb);
      } else {
        const CUtensorMap* map = &tm.m[it.slot][up ? 0 : 1];
        const uint32_t tile = up ? 8u * rowb : 16u * rowb;  // bytes of one tile box
        for (int m = 0; m < n; ++m) {
          if (up) {
            tma3d(smem_u32(ring + d.w0 + m * tile), map, 0, (int)(row0 + 8 * (rb0 + m)), 0, &full[s]);
            tma3d(smem_u32(ring + d.w1 + m * tile), map, 0, (int)(row0 + p.I + 8 * (rb0 + m)), 0, &full[s]);
          } else {
            tma3d(smem_u32(ring + d.w0 + m * tile), map, 0, (int)(row0 + 16 * (rb0 + m)), 0, &full[s]);
          }
        }
      }
      if (up) {
        if (sb) {
          bulk_g2s(ring + d.s0, sc + (size_t)8 * rb0 * srow, sb / 2, &full[s]);
          bulk_g2s(ring + d.s1, sc + (size_t)(p.I + 8 * rb0) * srow, sb / 2, &full[s]);
        }
        if (fresh) {
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if (j < it.ntok)
              bulk_g2s(ring + d.xo + (uint32_t)j * K * 2u, static_cast<const uint8_t*>(p.x) + (size_t)tok[j] * p.H * 2,
                       (uint32_t)K * 2u, &full[s]);
        }
      } else {
        if (sb) bulk_g2s(ring + d.s0, sc + (size_t)16 * rb0 * srow, sb, &full[s]);
        if (fresh) {
          // the item's h rows exist once every gate/up unit of the item has finished
          ok = wait_counter(p.updone + item, Uup, p.status);
          if (ok) {
            asm volatile("fence.proxy.async.global;" ::: "memory");
            bulk_g2s(ring + d.xo, static_cast<const uint8_t*>(p.h) + (size_t)it.start * p.I * 2, xb, &full[s]);
          } else {
            // give up: the slot completes once its weight copies land and tells the consumers to stop
            mbar_complete_tx(&full[s], xb);
            d.item = -1;
          }
        }
      }
      mbar_arrive1(&full[s]);
      ++seq;
      cur += n;
      if (!ok) break;
    }
    if (ok && free_until(0)) {
      const uint32_t s = seq % kDecSlots;
      jobs[s].item = -1;
      mbar_arrive1(&full[s]);
      ++seq;
    }
    // the CTA must not retire with copies in flight (they complete the jobs' full barriers)
    for (uint32_t j = oldest; j < seq; ++j) mbar_wait(&full[j % kDecSlots], (j / kDecSlots) & 1, nullptr);
    return;
  }

  if (warp == kDecEpi) {
    // ======================= epilogue warp =======================
    int pend_item[kDecRed], pend_n[kDecRed];
    int np = 0, since = 0;  // pending distinct items; gate/up jobs since the last flush
    bool zero_seen = false, ok = true;
    int cur_item = -1, cur_up = -1;
    int etok[2] = {0, 0};
    float ew[2] = {0.f, 0.f};
    auto flush = [&]() {
      // h of the pending gate/up jobs -> visible to every CTA (and to its bulk copies), then counted
      __threadfence();
      asm volatile("fence.proxy.async.global;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
#pragma unroll
        for (int j = 0; j < kDecRed; ++j)
          if (j < np) atomicAdd(p.updone + pend_item[j], pend_n[j]);
      }
      np = 0;
      since = 0;
    };
    for (uint32_t seq = 0;; ++seq) {
      const int b = seq % kDecRed;
      const uint32_t par = (seq / kDecRed) & 1;
      // wait for the job's sums; counts still pending are published when a wait runs past ~1 us
      // (a CTA elsewhere may be waiting for them)
      bool got = false;
      const uint64_t t_wait = gtime();
      for (uint32_t i = 0; i < kSpinLimit; ++i) {
        int r = 0, fl = 0;
        if (lane == 0) {
          r = mbar_try_wait(&sums_ready[b], par);
          fl = !r && np > 0 && gtime() - t_wait > 1000;
        }
        if (__shfl_sync(0xffffffffu, r, 0)) {
          got = true;
          break;
        }
        if (__shfl_sync(0xffffffffu, fl, 0)) flush();
      }
      if (!got) {
        if (lane == 0) atomicExch(p.status, kDevTimeout);
        ok = false;
        break;
      }
      const RedHdr hd = hdr[b];
      if (hd.item < 0) break;
      if (!hd.up && np > 0) flush();  // this CTA's gate/up jobs are over: publish their counts now
      // the consumers' partial sums, added in warp order (the same sum on every run)
      float vs[kDecMT][4];
#pragma unroll
      for (int m = 0; m < kDecMT; ++m)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          vs[m][e] = 0.f;
          if (m < hd.n) {
            const float* a = red + b * kRedFloats + (m * 4 + e) * 32 + lane;
#pragma unroll
            for (int w = 0; w < kDecCons; ++w) vs[m][e] += a[w * kRedSlice];
          }
        }
      __syncwarp();
      if (lane == 0) mbar_arrive1(&buf_free[b]);  // buffer b now takes job seq + kDecRed
      if (hd.item != cur_item || hd.up != cur_up) {
        cur_item = hd.item;
        cur_up = hd.up;
        if (!hd.up) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int tk = 2 * t + e;
            if (tk < hd.ntok) {
              const int ps = __ldg(p.pos + hd.start + tk);
              etok[e] = ps / p.k;
              ew[e] = __ldg(p.wflat + ps);
            }
          }
        }
      }
      if (hd.up) {
        AT* hp = static_cast<AT*>(p.h);
#pragma unroll
        for (int m = 0; m < kDecMT; ++m)
          if (m < hd.n) {
            const int r = 8 * (hd.rb0 + m) + g;
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int tk = 2 * t + e;
              if (tk < hd.ntok) hp[(int64_t)(hd.start + tk) * p.I + r] = from_f32<AT>(silu_mul(vs[m][e], vs[m][2 + e]));
            }
          }
        // count the job now or with the next jobs (one fence for all of them)
        bool merged = false;
#pragma unroll
        for (int j = 0; j < kDecRed; ++j)
          if (j < np && pend_item[j] == hd.item) {
            pend_n[j] += hd.n;
            merged = true;
          }
        if (!merged) {
#pragma unroll
          for (int j = 0; j < kDecRed; ++j)
            if (j == np) {
              pend_item[j] = hd.item;
              pend_n[j] = hd.n;
            }
          ++np;
        }
        // publish at least every 2 kDecRed gate/up jobs, so down jobs elsewhere are not held back
        if (np == kDecRed || ++since >= 2 * kDecRed) flush();
      } else {
        if (!zero_seen) {  // every CTA has cleared its part of acc
          bool zok = true;
          if (lane == 0) zok = wait_counter(p.ctr + 1, (int32_t)gridDim.x, p.status);
          if (!__shfl_sync(0xffffffffu, (int)zok, 0)) {
            ok = false;
            break;
          }
          zero_seen = true;
        }
#pragma unroll
        for (int m = 0; m < kDecMT; ++m)
          if (m < hd.n) {
            const int r = 16 * (hd.rb0 + m) + g;
#pragma unroll
            for (int e = 0; e < 2; ++e)
              if (2 * t + e < hd.ntok) {
                float* arow = p.acc + (int64_t)etok[e] * p.H + r;
                red_add_f32(arow, ew[e] * vs[m][e]);
                red_add_f32(arow + 8, ew[e] * vs[m][2 + e]);
              }
          }
      }
    }
    if (np > 0) flush();
    if (!ok || !p.out) return;
    // every CTA's reductions are in acc once all CTAs have counted themselves done
    __threadfence();
    __syncwarp();
    bool dok = true;
    if (lane == 0) {
      atomicAdd(p.ctr + 2, 1);
      dok = wait_counter(p.ctr + 2, (int32_t)gridDim.x, p.status);
    }
    if (!__shfl_sync(0xffffffffu, (int)dok, 0)) return;
    __threadfence();
    // this CTA's slice of the output, 4 elements per lane step
    const int64_t n4 = (int64_t)p.T * p.H / 4;
    const int64_t per = (n4 + gridDim.x - 1) / gridDim.x;
    const int64_t lo = (int64_t)blockIdx.x * per, hi = min64(n4, lo + per);
    AT* o = static_cast<AT*>(p.out);
    for (int64_t i = lo + lane; i < hi; i += 32) {
      const float4 a = __ldcg(reinterpret_cast<const float4*>(p.acc) + i);
      float v[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (p.add) v[e] += to_f32<AT>(o[4 * i + e]);
        o[4 * i + e] = from_f32<AT>(v[e]);
      }
    }
    return;
  }

  // ======================= consumers =======================
  {
    // clear the combine buffer (and the output of a call without items), then count this CTA in
    const int64_t n = (int64_t)p.T * p.H;
    const int64_t stride = (int64_t)gridDim.x * (kDecCons * 32);
    for (int64_t i = (int64_t)blockIdx.x * (kDecCons * 32) + threadIdx.x; i < n; i += stride) p.acc[i] = 0.f;
    if (n_items == 0 && p.out && !p.add)
      for (int64_t i = (int64_t)blockIdx.x * (kDecCons * 32) + threadIdx.x; i < n; i += stride)
        static_cast<AT*>(p.out)[i] = from_f32<AT>(0.f);
    __threadfence();
    asm volatile("bar.sync 1, %0;" ::"n"(kDecCons * 32) : "memory");
    if (threadIdx.x == 0) atomicAdd(p.ctr + 1, 1);
  }
  uint32_t B[kDecCmax][8];
  float corr[kDecCmax][2];
  int kind = kKF;
  for (uint32_t seq = 0;; ++seq) {
    const uint32_t s = seq % kDecSlots;
    const int b = seq % kDecRed;
    if (!mbar_wait(&full[s], (seq / kDecSlots) & 1, p.status)) break;
    const DecJob d = jobs[s];
    if (d.item < 0) {
      // tell the epilogue warp that no job follows: a header with item -1 in the next buffer
      if (lane == 0) {
        if (seq >= kDecRed) mbar_wait(&buf_free[b], ((seq / kDecRed) - 1) & 1, p.status);
        if (warp == 0) hdr[b].item = -1;
        mbar_arrive1(&sums_ready[b]);
      }
      break;
    }
    const bool up = d.up != 0;
    const int K = up ? p.H : p.I;
    const int nch = K / 64;
    const int c0 = nch * warp / kDecCons, nc = nch * (warp + 1) / kDecCons - c0;
    if (d.fresh) {
      const int wt = p.lay[d.slot].wtype;
      kind = wt == MOEB200_I4 ? kKI4 : wt == MOEB200_I8 ? kKI8 : kKF;
      load_operand<AT>(ring + d.xo + (uint32_t)g * K * 2u, g < d.ntok, kind, c0, nc, g, t, B, corr);
    }
    const uint32_t rowb = (uint32_t)(K * gemv_wbits(p.lay[d.slot].wtype) / 8);
    const uint32_t srow = (uint32_t)(K / 64) * 2u;
    // tile m's box: gate/up = 8 gate rows at w0 (and 8 up rows at w1), down = 16 rows at w0; the lane
    // reads rows g and g+8 (gate/up: row g of the gate box and of the up box)
    const int R = up ? 8 : 16;
    const uint32_t tile = (uint32_t)R * rowb;
    const uint8_t* rg0 = ring + d.w0 + (uint32_t)g * 128u;
    const uint8_t* rh0 = up ? ring + d.w1 + (uint32_t)g * 128u : ring + d.w0 + (uint32_t)(g + 8) * 128u;
    // scale rows of rows g and g+8 of tile 0; tile m's are m * sstep further
    const uint8_t* sg0 = ring + d.s0 + (uint32_t)g * srow;
    const uint8_t* sh0 = ring + d.s1 + (uint32_t)(up ? g : g + 8) * srow;
    const uint32_t sstep = (uint32_t)(up ? 8 : 16) * srow;
    // the lane's bytes of each of the warp's groups, from a row base (swz_off without the row part)
    uint32_t colo[kDecCmax];
#pragma unroll
    for (int cl = 0; cl < kDecCmax; ++cl) {
      const int c = c0 + cl;
      const int bb = kind == kKI4 ? c * 32 + t * 8 : kind == kKI8 ? c * 64 + t * 16 : c * 128 + t * 32;
      colo[cl] = swz_off(R, g, bb) - (uint32_t)g * 128u;
    }
    float* rb = red + b * kRedFloats + warp * kRedSlice;
    const bool ok = consume<AT>(kind, d.n, rg0, rh0, tile, sg0, sh0, sstep, c0, nc, colo, B, corr, lane, &empty[s],
                                &buf_free[b], seq, rb, p.status);
    if (!ok) break;
    if (warp == 0 && lane == 0) {  // what the epilogue warp needs of the job
      RedHdr h;
      h.item = d.item;
      h.up = d.up;
      h.rb0 = d.rb0;
      h.n = d.n;
      h.start = d.start;
      h.ntok = d.ntok;
      h._pad[0] = h._pad[1] = 0;
      hdr[b] = h;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive1(&sums_ready[b]);
  }
}

}  // namespace

bool decode_supported(const moeb200_layout* lays, int nlay, int act_type, int H, int I) {
  if (act_type != MOEB200_F16 && act_type != MOEB200_BF16) return false;
  if (H % 64 || I % 64 || H < 64 || I < 64) return false;
  if (H / 64 > kDecCmax * kDecCons || I / 64 > kDecCmax * kDecCons) return false;
  uint32_t max_unit = 0;
  for (int i = 0; i < nlay; ++i) {
    const moeb200_layout& L = lays[i];
    const bool isint = L.wtype == MOEB200_I4 || L.wtype == MOEB200_I8;
    if (isint && (L.gs_up != 64 || L.gs_dn != 64)) return false;
    if (!isint && L.wtype != act_type) return false;
    const uint32_t bits = gemv_wbits(L.wtype);
    const uint32_t rb_up = (uint32_t)H * bits / 8, rb_dn = (uint32_t)I * bits / 8;
    // tensor-map rows: whole 128-byte segments, pitches that divide the record alignment and the
    // field offsets (records are 4096-byte aligned above the maps' base)
    if (rb_up % 128 || rb_dn % 128 || 4096 % rb_up || 4096 % rb_dn) return false;
    if (L.off_gu_q % rb_up || L.off_dn_q % rb_dn) return false;
    max_unit = std::max<uint32_t>(max_unit, 16u * rb_up + 16u * (H / 64) * 2);
    max_unit = std::max<uint32_t>(max_unit, 16u * rb_dn + 16u * (I / 64) * 2);
  }
  // a job of one unit plus the activation rows of 8 tokens must fit the ring
  return max_unit + 8u * (uint32_t)std::max(H, I) * 2u + 3 * 1024 <= (uint32_t)kDecRing;
}

cudaError_t launch_decode(const DecodeParams& p, const moeb200_layout* lays, int nlay, int act_type, int grid,
                          cudaStream_t s) {
  DecMaps tm{};
  for (int i = 0; i < nlay; ++i) {
    const int bits = gemv_wbits(lays[i].wtype);
    cudaError_t e = tma_rows3d_map(&tm.m[i][0], (uint64_t)p.tma_base, p.H * bits / 8, 8);
    if (e != cudaSuccess) return e;
    e = tma_rows3d_map(&tm.m[i][1], (uint64_t)p.tma_base, p.I * bits / 8, 16);
    if (e != cudaSuccess) return e;
  }
  if (act_type == MOEB200_BF16) {
    cudaError_t e = cudaFuncSetAttribute(decode_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, kDecSmem);
    if (e != cudaSuccess) return e;
    return launch_chained(decode_kernel<__nv_bfloat16>, dim3(grid), dim3(kDecThreads), (size_t)kDecSmem, s, p, tm);
  }
  cudaError_t e = cudaFuncSetAttribute(decode_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, kDecSmem);
  if (e != cudaSuccess) return e;
  return launch_chained(decode_kernel<__half>, dim3(grid), dim3(kDecThreads), (size_t)kDecSmem, s, p, tm);
}

}  // namespace moeb200
