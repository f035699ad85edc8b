// Grouped expert GEMM on the 5th-generation tensor cores -- the prefill path of the MoE layer.
//
// Replaces the reference's prefill expert path (moelab/runtime.py:335-355 `_accumulate`: per expert
// `materialize` (store.py:164-174) then two F.linear and an index_add) with two persistent kernels:
//
//   up   : D_gate[r, j], D_up[r, j] = sum_c W[r, c] * x[tok_j, c]    (two 128 x N tcgen05 MMAs per k-step)
//          h[j, r] = silu(D_gate) * D_up                              (epilogue, stored in the activation type)
//   down : D[r, j] = sum_c Wd[r, c] * h[j, c];  acc[tok_j, r] += w_j * D[r, j]   (fp32 reduction = combine)
//
// A tile is (work item, 128 weight rows); an item holds up to 128 routed pairs of one (expert,
// precision), so N = pairs rounded up to 16. Roles per CTA (one CTA per SM, persistent):
//   warps 0-7  dequantise the int4/int8/float record rows of each 64-column k-block into bf16/fp16
//              in 128-byte-swizzled K-major shared tiles, with the same rounding as moelab's
//              materialize in the activation dtype: (q - 8) exact, times the fp16 scale converted to
//              the activation type, one rounding;
//   warp 12    gathers the N token rows (or h rows) of each k-block with cp.async into the B tile;
//   warp 13    allocates TMEM and issues tcgen05.mma (kind::f16, fp32 accumulate) from one thread,
//              committing each stage back to the producers and each finished tile to the epilogue;
//   warps 8-11 read the accumulators with tcgen05.ld (double-buffered TMEM) and run the epilogue.
// Every wait is bounded (status word + early exit), the TMEM is freed on every path.
#include <type_traits>

#include "gemv.cuh"

namespace moeb200 {

namespace {

constexpr int BM = 128;          // weight rows per tile (MMA M)
constexpr int BK = 64;           // k-block: one 128-byte swizzle row of 16-bit values
constexpr int NMAX = 128;        // max tokens per item (MMA N)
constexpr int kThreads = 14 * 32;
constexpr int kDqWarps = 8;
constexpr int kEpiWarp0 = 8;
constexpr int kLoadWarp = 12;
constexpr int kMmaWarp = 13;
constexpr int kTileBytes = BM * 128;  // one 128 x 64 16-bit tile = 16 KB (also the B tile)

template <bool UP>
struct Geo {
  static constexpr int NA = UP ? 2 : 1;               // A tiles per stage (gate + up)
  static constexpr int STAGES = UP ? 4 : 6;
  static constexpr int STAGE_BYTES = (NA + 1) * kTileBytes;
  static constexpr int TMEM_COLS = UP ? 512 : 256;    // two accumulator buffers
  static constexpr int BUF_COLS = UP ? 256 : 128;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

// ---- tcgen05 / proxy primitives -----------------------------------------------------------------
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// SW128 K-major UMMA shared-memory descriptor: rows of 128 bytes, 8-row atoms 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;              // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024u >> 4) << 32;    // stride byte offset: next 8-row group
  d |= (uint64_t)1u << 46;              // descriptor version (sm_100)
  d |= (uint64_t)2u << 61;              // SWIZZLE_128B
  return d;
}

// kind::f16 instruction descriptor: fp32 accumulator, A/B fp16 or bf16, both K-major, M=128.
__device__ __forceinline__ uint32_t idesc_f16(bool bf16, int n) {
  const uint32_t fmt = bf16 ? 1u : 0u;
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t dtmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(dtmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint4 ldg16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

__device__ __forceinline__ void sts16(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}

// byte address of 16-byte chunk c (0..7) of row r in a 1024-byte-aligned SW128 tile
__device__ __forceinline__ uint32_t swz(uint32_t tile, int r, int c) { return tile + r * 128 + ((c ^ (r & 7)) << 4); }

// ---- dequantisation of 8 consecutive columns into 8 16-bit values (natural order) -----------------
template <typename AT>
__device__ __forceinline__ uint32_t mul2(uint32_t a, uint32_t s2);
template <>
__device__ __forceinline__ uint32_t mul2<__half>(uint32_t a, uint32_t s2) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(s2));
  return r;
}
template <>
__device__ __forceinline__ uint32_t mul2<__nv_bfloat16>(uint32_t a, uint32_t s2) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(s2));
  return r;
}

// scale (fp16 bits) -> activation-type pair (s, s), rounded like scales.to(dtype)
template <typename AT>
__device__ __forceinline__ uint32_t scale2(uint16_t s16) {
  const float f = __half2float(__ushort_as_half(s16));
  const AT a = from_f32<AT>(f);
  const uint16_t b = *reinterpret_cast<const uint16_t*>(&a);
  return (uint32_t)b | ((uint32_t)b << 16);
}

// int4 word (8 nibbles, columns c..c+7) -> 4 natural pairs times the scale
template <typename AT>
__device__ __forceinline__ void dq_int4_chunk(uint32_t w, uint32_t s2, uint32_t (&o)[4]) {
  uint32_t p04, p15, p26, p37;
  Dq<AT>::int4x8(w, p04, p15, p26, p37);  // exact (q-8) pairs (c,c+4) (c+1,c+5) (c+2,c+6) (c+3,c+7)
  o[0] = mul2<AT>(prmt(p04, p15, 0x5410), s2);  // (c, c+1)
  o[1] = mul2<AT>(prmt(p26, p37, 0x5410), s2);  // (c+2, c+3)
  o[2] = mul2<AT>(prmt(p04, p15, 0x7632), s2);  // (c+4, c+5)
  o[3] = mul2<AT>(prmt(p26, p37, 0x7632), s2);  // (c+6, c+7)
}

template <typename AT>
__device__ __forceinline__ void dq_int8_chunk(uint32_t w0, uint32_t w1, uint16_t s16, uint32_t (&o)[4]) {
  if constexpr (std::is_same<AT, __half>::value) {
    const uint32_t s2 = scale2<AT>(s16);
    uint32_t a, b, c, d;
    Dq<AT>::int8x4(w0, a, b);
    Dq<AT>::int8x4(w1, c, d);
    o[0] = mul2<AT>(a, s2);
    o[1] = mul2<AT>(b, s2);
    o[2] = mul2<AT>(c, s2);
    o[3] = mul2<AT>(d, s2);
  } else {
    // bf16: q * bf16(s) is exact in fp32 (8-bit by 8-bit), one rounding to bf16
    const float s = __bfloat162float(__float2bfloat16_rn(__half2float(__ushort_as_half(s16))));
    const uint32_t ws[2] = {w0, w1};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int32_t v = (int32_t)ws[h];
      const float q0 = (float)(int8_t)(v & 0xff), q1 = (float)(int8_t)((v >> 8) & 0xff);
      const float q2 = (float)(int8_t)((v >> 16) & 0xff), q3 = (float)(int8_t)((v >> 24) & 0xff);
      o[2 * h] = Dq<AT>::pack_f32(q0 * s, q1 * s);
      o[2 * h + 1] = Dq<AT>::pack_f32(q2 * s, q3 * s);
    }
  }
}

// ---- kernel -------------------------------------------------------------------------------------------
struct TcTile;
template <typename AT, bool UP, int STAGES, int STAGE_BYTES>
__device__ __forceinline__ bool dq_int4_tile(const TcTile& d, int nkb, int tile_i, int row, int c0, uint32_t& st,
                                             uint32_t sbase, uint64_t* empty, uint64_t* full_a, int32_t* status,
                                             int lane);

struct TcTile {
  int item, r0, ntok, n, start, slot;
  const uint8_t* q[2];  // first weight row of each A tile
  const uint8_t* s[2];  // first scale row of each A tile (integer records)
  int64_t rstride;
  int sstride, gs, wtype;
};

template <bool UP>
__device__ __forceinline__ void tc_describe(const GemvParams& p, int tile, int rb_per_item, TcTile& d) {
  d.item = tile / rb_per_item;
  const int rb = tile % rb_per_item;
  const Item it = p.items[d.item];
  const LayoutDev L = p.lay[it.slot];
  d.slot = it.slot;
  d.ntok = it.ntok;
  d.n = (it.ntok + 15) & ~15;
  d.start = it.start;
  d.r0 = rb * BM;
  d.wtype = L.wtype;
  const int K = UP ? p.H : p.I;
  const int wb = L.wtype == MOEB200_I4 ? 4 : L.wtype == MOEB200_I8 ? 8 : L.wtype == MOEB200_F32 ? 32 : 16;
  d.rstride = (int64_t)K * wb / 8;
  d.gs = UP ? L.gs_up : L.gs_dn;
  const bool isint = L.wtype == MOEB200_I4 || L.wtype == MOEB200_I8;
  d.sstride = isint ? (K / d.gs) * 2 : 0;
  const uint8_t* q = reinterpret_cast<const uint8_t*>(UP ? it.p_guq : it.p_dnq);
  const uint8_t* s = reinterpret_cast<const uint8_t*>(UP ? it.p_gus : it.p_dns);
  d.q[0] = q + (int64_t)d.r0 * d.rstride;
  d.s[0] = s + (int64_t)d.r0 * d.sstride;
  if (UP) {
    d.q[1] = q + (int64_t)(p.I + d.r0) * d.rstride;
    d.s[1] = s + (int64_t)(p.I + d.r0) * d.sstride;
  } else {
    d.q[1] = d.q[0];
    d.s[1] = d.s[0];
  }
}

// Raw source bytes of one thread's slice of a k-block (up to 128 bytes = 8 x 16).
struct Raw {
  uint4 v[8];
};

// UP: thread = one full row (8 chunks) of tile (warp / 4). DOWN: thread = half a row (4 chunks).
template <bool UP>
__device__ __forceinline__ void dq_coords(int dq_tid, int& tile, int& row, int& c0, int& nch) {
  if (UP) {
    tile = dq_tid >> 7;
    row = dq_tid & 127;
    c0 = 0;
    nch = 8;
  } else {
    tile = 0;
    row = dq_tid >> 1;
    c0 = (dq_tid & 1) * 4;
    nch = 4;
  }
}

template <bool UP>
__device__ __forceinline__ void dq_load(const TcTile& d, int kb, int tile, int row, int c0, Raw& raw) {
  const uint8_t* rowp = d.q[tile] + (int64_t)row * d.rstride;
  constexpr int NCH = UP ? 8 : 4;
  switch (d.wtype) {
    case MOEB200_I4: {  // 4 bytes per chunk
      const uint8_t* src = rowp + kb * 32 + c0 * 4;
#pragma unroll
      for (int i = 0; i < NCH / 4; ++i) raw.v[i] = ldg16(src + 16 * i);
      break;
    }
    case MOEB200_I8: {  // 8 bytes per chunk
      const uint8_t* src = rowp + kb * 64 + c0 * 8;
#pragma unroll
      for (int i = 0; i < NCH / 2; ++i) raw.v[i] = ldg16(src + 16 * i);
      break;
    }
    case MOEB200_F32: {  // 32 bytes per chunk: loaded and converted in dq_store
      break;
    }
    default: {  // 16-bit floats: 16 bytes per chunk
      const uint8_t* src = rowp + kb * 128 + c0 * 16;
#pragma unroll
      for (int i = 0; i < NCH; ++i) raw.v[i] = ldg16(src + 16 * i);
      break;
    }
  }
}

template <typename AT, bool UP>
__device__ __forceinline__ void dq_store(const TcTile& d, int kb, int tile, int row, int c0, const Raw& raw,
                                         uint32_t atile) {
  constexpr int NCH = UP ? 8 : 4;
  const bool isint = d.wtype == MOEB200_I4 || d.wtype == MOEB200_I8;
  const uint16_t* srow = isint ? reinterpret_cast<const uint16_t*>(d.s[tile] + (int64_t)row * d.sstride) : nullptr;
#pragma unroll
  for (int ci = 0; ci < NCH; ++ci) {
    const int c = c0 + ci;
    uint32_t o[4];
    if (d.wtype == MOEB200_I4) {
      const uint32_t* wv = reinterpret_cast<const uint32_t*>(&raw.v[ci / 4]);
      const uint16_t s16 = __ldg(srow + (kb * BK + c * 8) / d.gs);
      dq_int4_chunk<AT>(wv[ci % 4], scale2<AT>(s16), o);
    } else if (d.wtype == MOEB200_I8) {
      const uint32_t* wv = reinterpret_cast<const uint32_t*>(&raw.v[ci / 2]);
      const uint16_t s16 = __ldg(srow + (kb * BK + c * 8) / d.gs);
      dq_int8_chunk<AT>(wv[(ci % 2) * 2], wv[(ci % 2) * 2 + 1], s16, o);
    } else if (d.wtype == MOEB200_F32) {
      const float* f = reinterpret_cast<const float*>(d.q[tile] + (int64_t)row * d.rstride) + kb * BK + c * 8;
      const float4 a = __ldg(reinterpret_cast<const float4*>(f));
      const float4 b = __ldg(reinterpret_cast<const float4*>(f + 4));
      o[0] = Dq<AT>::pack_f32(a.x, a.y);
      o[1] = Dq<AT>::pack_f32(a.z, a.w);
      o[2] = Dq<AT>::pack_f32(b.x, b.y);
      o[3] = Dq<AT>::pack_f32(b.z, b.w);
    } else {
      const uint32_t* wv = reinterpret_cast<const uint32_t*>(&raw.v[ci]);
      const bool same = (d.wtype == MOEB200_F16) == std::is_same<AT, __half>::value;
      if (same) {
        o[0] = wv[0];
        o[1] = wv[1];
        o[2] = wv[2];
        o[3] = wv[3];
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float lo, hi;
          if (d.wtype == MOEB200_F16) {
            lo = __half2float(__ushort_as_half((uint16_t)(wv[i] & 0xffff)));
            hi = __half2float(__ushort_as_half((uint16_t)(wv[i] >> 16)));
          } else {
            lo = __uint_as_float(wv[i] << 16);
            hi = __uint_as_float(wv[i] & 0xffff0000u);
          }
          o[i] = Dq<AT>::pack_f32(lo, hi);
        }
      }
    }
    sts16(swz(atile, row, c), o[0], o[1], o[2], o[3]);
  }
}

// int4 records whose groups span whole 64-column k-blocks: the thread's raw bytes are loaded two to
// three k-blocks ahead of their dequantisation, one scale per row per k-block.
template <typename AT, bool UP, int STAGES, int STAGE_BYTES>
__device__ __forceinline__ bool dq_int4_tile(const TcTile& d, int nkb, int tile_i, int row, int c0, uint32_t& st,
                                             uint32_t sbase, uint64_t* empty, uint64_t* full_a, int32_t* status,
                                             int lane) {
  constexpr int NV = UP ? 2 : 1;   // 16-byte vectors per k-block (32 or 16 raw bytes)
  constexpr int NCH = UP ? 8 : 4;  // 8-column chunks per k-block
  const uint8_t* rowp = d.q[tile_i] + (int64_t)row * d.rstride + c0 * 4;
  const uint16_t* srow = reinterpret_cast<const uint16_t*>(d.s[tile_i] + (int64_t)row * d.sstride);
  const int kpg = d.gs / BK;  // k-blocks per scale group
  constexpr int MB = 2;       // k-blocks per prefetch macro block
  uint4 raw[MB][NV], nraw[MB][NV];
  uint16_t sc[MB], nsc[MB];
#pragma unroll
  for (int u = 0; u < MB; ++u) {
#pragma unroll
    for (int i = 0; i < NV; ++i) raw[u][i] = ldg16(rowp + u * 32 + i * 16);
    sc[u] = __ldg(srow + u / kpg);
  }
  for (int kb0 = 0; kb0 < nkb; kb0 += MB) {
    const bool more = kb0 + MB < nkb;
    if (more) {
#pragma unroll
      for (int u = 0; u < MB; ++u) {
#pragma unroll
        for (int i = 0; i < NV; ++i) nraw[u][i] = ldg16(rowp + (kb0 + MB + u) * 32 + i * 16);
        nsc[u] = __ldg(srow + (kb0 + MB + u) / kpg);
      }
    }
#pragma unroll
    for (int u = 0; u < MB; ++u, ++st) {
      const int s = st % STAGES;
      if (!mbar_wait(&empty[s], ((st / STAGES) & 1u) ^ 1u, status)) return false;
      const uint32_t atile = sbase + s * STAGE_BYTES + tile_i * kTileBytes;
      const uint32_t s2 = scale2<AT>(sc[u]);
#pragma unroll
      for (int ci = 0; ci < NCH; ++ci) {
        const uint32_t* wv = reinterpret_cast<const uint32_t*>(&raw[u][ci / 4]);
        uint32_t o[4];
        dq_int4_chunk<AT>(wv[ci % 4], s2, o);
        sts16(swz(atile, row, c0 + ci), o[0], o[1], o[2], o[3]);
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full_a[s]);
    }
    if (more) {
#pragma unroll
      for (int u = 0; u < MB; ++u) {
#pragma unroll
        for (int i = 0; i < NV; ++i) raw[u][i] = nraw[u][i];
        sc[u] = nsc[u];
      }
    }
  }
  return true;
}

template <typename AT, bool UP>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_kernel(const GemvParams p) {
  using G = Geo<UP>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - smem_u32(smem_raw));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sgen + G::STAGES * G::STAGE_BYTES);
  uint64_t* full_a = bars;                     // [STAGES] 8 dequant-warp arrivals
  uint64_t* full_b = bars + G::STAGES;         // [STAGES] 1 loader arrival
  uint64_t* empty = bars + 2 * G::STAGES;      // [STAGES] 1 tcgen05.commit
  uint64_t* acc_full = bars + 3 * G::STAGES;   // [2] 1 tcgen05.commit
  uint64_t* acc_empty = acc_full + 2;          // [2] 4 epilogue-warp arrivals
  uint64_t* done_bar = acc_empty + 2;          // [1] final commit before freeing TMEM
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (UP && p.zero_acc) {
    const int64_t n = (int64_t)p.T * p.H;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
      p.acc[i] = 0.f;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < G::STAGES; ++s) {
      mbar_init(&full_a[s], kDqWarps);
      mbar_init(&full_b[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(done_bar, 1);
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "n"(G::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int n_items = *p.n_items;
  const int rb_per_item = (UP ? p.I : p.H) / BM;
  const int n_tiles = n_items * rb_per_item;
  const int nkb = (UP ? p.H : p.I) / BK;
  bool ok = true;

  if (warp < kDqWarps) {
    // ---------------- dequant producers ----------------
    int tile_i, row, c0, nch;
    dq_coords<UP>(threadIdx.x, tile_i, row, c0, nch);
    uint32_t st = 0;
    for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
      TcTile d;
      tc_describe<UP>(p, tile, rb_per_item, d);
      if (d.wtype == MOEB200_I4 && d.gs % BK == 0 && nkb % 2 == 0) {
        if (!dq_int4_tile<AT, UP, G::STAGES, G::STAGE_BYTES>(d, nkb, tile_i, row, c0, st, sbase, empty, full_a,
                                                             p.status, lane)) {
          ok = false;
          break;
        }
        continue;
      }
      Raw cur;
      dq_load<UP>(d, 0, tile_i, row, c0, cur);
      for (int kb = 0; kb < nkb; ++kb, ++st) {
        Raw nxt;
        if (kb + 1 < nkb) dq_load<UP>(d, kb + 1, tile_i, row, c0, nxt);
        const int s = st % G::STAGES;
        if (!mbar_wait(&empty[s], ((st / G::STAGES) & 1u) ^ 1u, p.status)) { ok = false; break; }
        const uint32_t atile = sbase + s * G::STAGE_BYTES + tile_i * kTileBytes;
        dq_store<AT, UP>(d, kb, tile_i, row, c0, cur, atile);
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_a[s]);
        if (kb + 1 < nkb) cur = nxt;
      }
    }
  } else if (warp == kLoadWarp) {
    // ---------------- B loader: token rows (up) or h rows (down), cp.async into SW128 tiles -------
    constexpr int LAG = G::STAGES - 2;
    uint32_t st = 0;
    uint32_t pending = 0;  // steps issued but not yet signalled
    for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
      TcTile d;
      tc_describe<UP>(p, tile, rb_per_item, d);
      // per-lane rows: lane handles rows lane, lane+32, ... of the N-row B tile
      const AT* rowp[NMAX / 32];
#pragma unroll
      for (int i = 0; i < NMAX / 32; ++i) {
        const int j = lane + 32 * i;
        if (j < d.ntok) {
          if (UP) {
            const int tok = p.pos[d.start + j] / p.k;
            rowp[i] = static_cast<const AT*>(p.x) + (int64_t)tok * p.H;
          } else {
            rowp[i] = static_cast<const AT*>(p.h) + (int64_t)(d.start + j) * p.I;
          }
        } else {
          rowp[i] = static_cast<const AT*>(UP ? p.x : p.h);  // zero-filled (src size 0)
        }
      }
      for (int kb = 0; kb < nkb; ++kb, ++st) {
        const int s = st % G::STAGES;
        if (!mbar_wait(&empty[s], ((st / G::STAGES) & 1u) ^ 1u, p.status)) { ok = false; break; }
        const uint32_t btile = sbase + s * G::STAGE_BYTES + G::NA * kTileBytes;
#pragma unroll
        for (int i = 0; i < NMAX / 32; ++i) {
          const int j = lane + 32 * i;
          if (j < d.n) {
            const uint32_t bytes = j < d.ntok ? 16u : 0u;
#pragma unroll
            for (int c = 0; c < 8; ++c) cp_async16(swz(btile, j, c), rowp[i] + kb * BK + c * 8, bytes);
          }
        }
        cp_async_commit();
        ++pending;
        if (pending > (uint32_t)LAG) {
          cp_async_wait<LAG>();
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) mbar_arrive(&full_b[(st - LAG) % G::STAGES]);
          --pending;
        }
      }
    }
    cp_async_wait<0>();
    fence_proxy_async();
    __syncwarp();
    if (lane == 0)
      for (uint32_t q = pending; q > 0; --q) mbar_arrive(&full_b[(st - q) % G::STAGES]);
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer (one thread) ----------------
    if (lane == 0) {
      uint32_t st = 0, tcount = 0;
      for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x, ++tcount) {
        TcTile d;
        tc_describe<UP>(p, tile, rb_per_item, d);
        const int buf = tcount & 1;
        if (!mbar_wait(&acc_empty[buf], ((tcount >> 1) & 1u) ^ 1u, p.status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t idesc = idesc_f16(std::is_same<AT, __nv_bfloat16>::value, d.n);
        const uint32_t d0 = tmem + buf * G::BUF_COLS;
        for (int kb = 0; kb < nkb; ++kb, ++st) {
          const int s = st % G::STAGES;
          const uint32_t par = (st / G::STAGES) & 1u;
          if (!mbar_wait(&full_a[s], par, p.status) || !mbar_wait(&full_b[s], par, p.status)) { ok = false; break; }
          tc_fence_after();
          const uint32_t stage = sbase + s * G::STAGE_BYTES;
          const uint32_t btile = stage + G::NA * kTileBytes;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t bdesc = sw128_desc(btile + kk * 32);
            const uint32_t accum = (kb > 0 || kk > 0) ? 1u : 0u;
            tc_mma(d0, sw128_desc(stage + kk * 32), bdesc, idesc, accum);
            if (UP) tc_mma(d0 + NMAX, sw128_desc(stage + kTileBytes + kk * 32), bdesc, idesc, accum);
          }
          tc_commit(&empty[s]);
        }
        if (!ok) break;
        tc_commit(&acc_full[buf]);
      }
      tc_commit(done_bar);
      mbar_wait(done_bar, 0, p.status);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue warps 8..11 ----------------
    const int q = warp - kEpiWarp0;  // TMEM lane quarter
    const int r_local = q * 32 + lane;
    uint32_t tcount = 0;
    for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x, ++tcount) {
      TcTile d;
      tc_describe<UP>(p, tile, rb_per_item, d);
      const int buf = tcount & 1;
      if (!mbar_wait(&acc_full[buf], (tcount >> 1) & 1u, p.status)) { ok = false; break; }
      tc_fence_after();
      const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + buf * G::BUF_COLS;
      const int row = d.r0 + r_local;
      for (int j0 = 0; j0 < d.n; j0 += 16) {
        uint32_t a[16];
        tmem_ld16(tb + j0, a);
        if (UP) {
          uint32_t u[16];
          tmem_ld16(tb + NMAX + j0, u);
          tmem_wait_ld();
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            const int j = j0 + jj;
            if (j < d.ntok) {
              const float hv = silu_mul(__uint_as_float(a[jj]), __uint_as_float(u[jj]));
              static_cast<AT*>(p.h)[(int64_t)(d.start + j) * p.I + row] = from_f32<AT>(hv);
            }
          }
        } else {
          tmem_wait_ld();
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            const int j = j0 + jj;
            if (j < d.ntok) {
              const int pos = p.pos[d.start + j];
              const int tok = pos / p.k;
              red_add_f32(p.acc + (int64_t)tok * p.H + row, p.wflat[pos] * __uint_as_float(a[jj]));
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(G::TMEM_COLS));
  }
}

template <typename AT, bool UP>
cudaError_t launch_tc_t(const GemvParams& p, int grid, cudaStream_t s) {
  auto kern = gemm_tc_kernel<AT, UP>;
  const int smem = Geo<UP>::SMEM;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, kThreads, smem, s>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemm_up(const GemvParams& p, int act_type, int grid, cudaStream_t s) {
  return act_type == MOEB200_BF16 ? launch_tc_t<__nv_bfloat16, true>(p, grid, s) : launch_tc_t<__half, true>(p, grid, s);
}

cudaError_t launch_gemm_down(const GemvParams& p, int act_type, int grid, cudaStream_t s) {
  return act_type == MOEB200_BF16 ? launch_tc_t<__nv_bfloat16, false>(p, grid, s)
                                  : launch_tc_t<__half, false>(p, grid, s);
}

}  // namespace moeb200
