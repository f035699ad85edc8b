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
// precision), so N = pairs rounded up to 16. One CTA per SM works through its tiles with five roles
// connected by shared-memory rings and mbarriers:
//   warp 22    (TMA producer) points a tensor map at each tile's record (tensormap.replace on the
//              device) and streams the tile's raw weight bytes through the RAW ring -- one unit is
//              128 bytes of each of the 128 (up: 2 x 128) rows, a 128-byte-swizzled TMA box -- and
//              the tile's whole scale rows into a double-buffered scale area (bulk copies). The ring
//              runs ahead across tile boundaries, so DRAM latency is hidden by the ring depth;
//   warps 0-15 dequantise each 64-column k-block from the raw ring into the A ring: 128-byte-swizzled
//              K-major bf16/fp16 tiles, with the rounding of moelab's materialize in the activation
//              dtype ((q - 8) exact, times the fp16 scale converted to the activation type, one
//              rounding; float records converted, or copied when the types agree);
//   warp 20    fills the B ring: the N token rows of the k-block gathered with cp.async (up), or one
//              TMA box of the item's contiguous h rows (down);
//   warp 21    allocates TMEM and issues tcgen05.mma (kind::f16, fp32 accumulate) from one thread,
//              committing each A and B stage back to its producer and each finished tile to the
//              epilogue (two TMEM accumulator buffers);
//   warps 16-19 read the accumulators with tcgen05.ld and run the epilogue (up: SwiGLU into h; down:
//              the router-weighted fp32 reduction into acc, token rows and weights of the tile held
//              in registers and broadcast with shuffles).
// Every wait is bounded (status word + early exit), copies in flight are waited for before exit,
// and the TMEM is freed on every path.
#include <algorithm>
#include <type_traits>

#include "gemv.cuh"
#include "tma.cuh"

namespace moeb200 {

namespace {

constexpr int BM = 128;          // weight rows per tile (MMA M)
constexpr int BK = 64;           // k-block: one 128-byte swizzle row of 16-bit values
constexpr int NMAX = 128;        // max tokens per item (MMA N)
constexpr int kDqWarps = 16;
constexpr int kEpiWarp0 = 16;  // epilogue warps 16..19: TMEM lane quarter = warp % 4
constexpr int kLoadWarp = 20;
constexpr int kMmaWarp = 21;
constexpr int kTmaWarp = 22;
constexpr int kThreads = 23 * 32;
constexpr int kTileBytes = BM * 128;  // one 128 x 64 16-bit operand tile = 128 rows x 128 raw bytes = 16 KB
constexpr int kMaxSmem = 227 * 1024;

// Tensor maps of a launch: per precision slot the phase's weight field (uint8 [rows][row bytes],
// 128 x 128 boxes, retargeted per tile), and for the down phase h [pairs][I] (64 x 128 boxes).
struct alignas(64) TcMaps {
  CUtensorMap w[4];
  CUtensorMap h;
};

// Ring depths and shared-memory offsets of a launch (planned on the host).
struct TcGeo {
  int32_t a_st, b_st, r_st;  // A (dequantised), B (tokens / h) and RAW ring depths
  int32_t lag;               // up: cp.async groups the B loader keeps in flight
  int32_t tmap_ring;         // tensor-map slots the producer cycles through (r_st + 1)
  uint32_t a_off, b_off, r_off, s_off, d_off, bar_off;
  uint32_t s_bytes;          // one scale buffer
};

// A ring cursor: slot and phase parity, advanced in the order every party walks the ring.
struct Ring {
  uint32_t slot = 0, phase = 0;
  __device__ __forceinline__ void next(int n) {
    if (++slot == (uint32_t)n) {
      slot = 0;
      phase ^= 1u;
    }
  }
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
// wait until at most n (0..4) of this thread's cp.async groups are pending
__device__ __forceinline__ void cp_async_wait_n(int n) {
  switch (n) {
    case 0: cp_async_wait<0>(); break;
    case 1: cp_async_wait<1>(); break;
    case 2: cp_async_wait<2>(); break;
    case 3: cp_async_wait<3>(); break;
    default: cp_async_wait<4>(); break;
  }
}

__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ uint16_t lds_u16(uint32_t a) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
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

// 8 16-bit record values (one 16-byte vector) in the activation type
template <typename AT, int WT>
__device__ __forceinline__ void cvt_f16x8(const uint4& v, uint32_t (&o)[4]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  constexpr bool same = (WT == MOEB200_F16) == std::is_same<AT, __half>::value;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (same) {
      o[i] = w[i];
    } else {
      float lo, hi;
      if constexpr (WT == MOEB200_F16) {
        lo = __half2float(__ushort_as_half((uint16_t)(w[i] & 0xffff)));
        hi = __half2float(__ushort_as_half((uint16_t)(w[i] >> 16)));
      } else {
        lo = __uint_as_float(w[i] << 16);
        hi = __uint_as_float(w[i] & 0xffff0000u);
      }
      o[i] = Dq<AT>::pack_f32(lo, hi);
    }
  }
}

// ---- tiles ----------------------------------------------------------------------------------------
struct TcTile {
  int item, r0, ntok, n, start, slot, wtype, gs, units, sstride;
  const uint8_t* q;  // weight field of the phase (float records: the matrix itself)
  const uint8_t* s;  // scale field (integer records)
};

__device__ __forceinline__ bool is_int_w(int wt) { return wt == MOEB200_I4 || wt == MOEB200_I8; }

template <bool UP>
__device__ __forceinline__ void tc_describe(const GemvParams& p, int tile, int rb_per_item, TcTile& d) {
  d.item = tile / rb_per_item;
  const int rb = tile - d.item * rb_per_item;
  const Item it = p.items[d.item];
  const LayoutDev L = p.lay[it.slot];
  d.slot = it.slot;
  d.ntok = it.ntok;
  d.n = (it.ntok + 15) & ~15;
  d.start = it.start;
  d.r0 = rb * BM;
  d.wtype = L.wtype;
  const int K = UP ? p.H : p.I;
  d.units = (K * gemv_wbits(L.wtype) / 8 + 127) >> 7;
  d.gs = UP ? L.gs_up : L.gs_dn;
  d.sstride = is_int_w(L.wtype) ? (K / d.gs) * 2 : 0;
  d.q = reinterpret_cast<const uint8_t*>(UP ? it.p_guq : it.p_dnq);
  d.s = reinterpret_cast<const uint8_t*>(UP ? it.p_gus : it.p_dns);
}

// Shared-memory rings of a CTA (shared-window addresses and barrier arrays).
struct Rings {
  uint32_t a, b, r, s, d;  // ring bases, scale areas, tensor-map staging
  uint64_t *afull, *aempty, *bfull, *bempty, *rfull, *rempty, *sfull, *sempty, *accf, *acce, *done;
  uint32_t* tmem_slot;
};

// ---- dequantisation of one tile: RAW ring -> A ring ------------------------------------------------
// Thread (part, row, c0): up: part 0/1 = gate/up rows, two threads per row (chunks c0..c0+3); down:
// four threads per row (chunks c0, c0+1). Sixteen warps keep enough independent dequantisation in
// flight: with eight, each warp's dependent chain of shared loads, conversions and stores (about 200
// instructions per k-block) set the pace at ~2,400 cycles per k-block, five times the MMA time.
// Units of the RAW ring are waited in order; a k-block lies in the last unit waited (16-bit and
// narrower records) or in the last two (fp32 records).
template <typename AT, bool UP, int WT>
__device__ __forceinline__ bool dq_tile(const TcTile& d, const TcGeo& g, const Rings& R, int nkb, int part, int row,
                                     int c0, uint32_t sarea, Ring& ar, Ring& rw, Ring& rr, int32_t* status,
                                     int lane) {
  constexpr int NA = UP ? 2 : 1;
  constexpr int WB = WT == MOEB200_I4 ? 4 : WT == MOEB200_I8 ? 8 : WT == MOEB200_F32 ? 32 : 16;
  constexpr int BPK = BK * WB / 8;  // raw bytes of a row per k-block
  constexpr int NCH = UP ? 4 : 2;   // 8-column chunks per thread and k-block
  constexpr int CB = WB;            // raw bytes of a chunk
  constexpr int NV = NCH * CB / 16; // 16-byte raw vectors per thread and k-block (int4 down: half of one)
  constexpr bool INT = WT == MOEB200_I4 || WT == MOEB200_I8;
  const uint32_t rslot = NA * kTileBytes;
  const uint32_t rrow = R.r + part * kTileBytes + row * 128;
  const uint32_t abase = R.a + part * kTileBytes;
  const int rsw = row & 7;
  const uint32_t srow = sarea + (part * BM + row) * d.sstride;
  const bool one_scale = INT && (d.gs % BK == 0);
  int waited = 0, released = 0;
  uint32_t cur = 0, prev = 0;  // RAW slot offsets of the last two units waited
  for (int kb = 0; kb < nkb; ++kb) {
    const int lo = kb * BPK;
    const int need = min(d.units, (lo + BPK + 127) >> 7);
    while (waited < need) {
      if (!mbar_wait(&R.rfull[rw.slot], rw.phase, status)) return false;
      prev = cur;
      cur = rw.slot * rslot;
      rw.next(g.r_st);
      ++waited;
    }
    if (!mbar_wait(&R.aempty[ar.slot], ar.phase ^ 1u, status)) return false;
    const uint32_t atile = abase + ar.slot * (NA * kTileBytes);
    uint32_t s2 = 0;
    uint16_t s16 = 0;
    if constexpr (INT) {
      if (one_scale) {
        s16 = lds_u16(srow + ((kb * BK) / d.gs) * 2);
        s2 = scale2<AT>(s16);
      }
    }
    auto raw = [&](int o) {  // 16 bytes at byte o of the row
      const uint32_t ub = ((o >> 7) == waited - 1) ? cur : prev;
      return lds128(rrow + ub + ((((o & 127) >> 4) ^ rsw) << 4));
    };
    if constexpr (WT == MOEB200_F32) {
#pragma unroll
      for (int ci = 0; ci < NCH; ++ci) {
        const int c = c0 + ci;
        const uint4 v0 = raw(lo + c * CB), v1 = raw(lo + c * CB + 16);
        sts16(swz(atile, row, c), Dq<AT>::pack_f32(__uint_as_float(v0.x), __uint_as_float(v0.y)),
              Dq<AT>::pack_f32(__uint_as_float(v0.z), __uint_as_float(v0.w)),
              Dq<AT>::pack_f32(__uint_as_float(v1.x), __uint_as_float(v1.y)),
              Dq<AT>::pack_f32(__uint_as_float(v1.z), __uint_as_float(v1.w)));
      }
    } else if constexpr (WT == MOEB200_I4 && NV == 0) {
      // two chunks = 8 bytes
      const int o = lo + c0 * CB;
      const uint32_t ub = ((o >> 7) == waited - 1) ? cur : prev;
      const uint2 v = lds64(rrow + ub + ((((o & 127) >> 4) ^ rsw) << 4) + (o & 15));
      const uint32_t w[2] = {v.x, v.y};
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int c = c0 + q;
        if (!one_scale) s2 = scale2<AT>(lds_u16(srow + ((kb * BK + c * 8) / d.gs) * 2));
        uint32_t out[4];
        dq_int4_chunk<AT>(w[q], s2, out);
        sts16(swz(atile, row, c), out[0], out[1], out[2], out[3]);
      }
    } else {
#pragma unroll
      for (int vi = 0; vi < NV; ++vi) {
        const uint4 v = raw(lo + c0 * CB + 16 * vi);
        if constexpr (WT == MOEB200_I4) {
          const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int c = c0 + vi * 4 + q;
            if (!one_scale) s2 = scale2<AT>(lds_u16(srow + ((kb * BK + c * 8) / d.gs) * 2));
            uint32_t out[4];
            dq_int4_chunk<AT>(w[q], s2, out);
            sts16(swz(atile, row, c), out[0], out[1], out[2], out[3]);
          }
        } else if constexpr (WT == MOEB200_I8) {
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const int c = c0 + vi * 2 + q;
            if (!one_scale) s16 = lds_u16(srow + ((kb * BK + c * 8) / d.gs) * 2);
            uint32_t out[4];
            dq_int8_chunk<AT>(q ? v.z : v.x, q ? v.w : v.y, s16, out);
            sts16(swz(atile, row, c), out[0], out[1], out[2], out[3]);
          }
        } else {
          uint32_t out[4];
          cvt_f16x8<AT, WT>(v, out);
          sts16(swz(atile, row, c0 + vi), out[0], out[1], out[2], out[3]);
        }
      }
    }
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) mbar_arrive(&R.afull[ar.slot]);
    ar.next(g.a_st);
    const int hi = lo + BPK;
    while (released < waited && ((released + 1) * 128 <= hi || kb == nkb - 1)) {
      if (lane == 0) mbar_arrive(&R.rempty[rr.slot]);
      rr.next(g.r_st);
      ++released;
    }
  }
  return true;
}


template <typename AT, bool UP>
__device__ __forceinline__ bool dq_dispatch(const TcTile& d, const TcGeo& g, const Rings& R, int nkb, int part, int row,
                                            int c0, uint32_t sarea, Ring& ar, Ring& rw, Ring& rr, int32_t* status,
                                            int lane) {
  switch (d.wtype) {
    case MOEB200_I4: return dq_tile<AT, UP, MOEB200_I4>(d, g, R, nkb, part, row, c0, sarea, ar, rw, rr, status, lane);
    case MOEB200_I8: return dq_tile<AT, UP, MOEB200_I8>(d, g, R, nkb, part, row, c0, sarea, ar, rw, rr, status, lane);
    case MOEB200_F16: return dq_tile<AT, UP, MOEB200_F16>(d, g, R, nkb, part, row, c0, sarea, ar, rw, rr, status, lane);
    case MOEB200_BF16:
      return dq_tile<AT, UP, MOEB200_BF16>(d, g, R, nkb, part, row, c0, sarea, ar, rw, rr, status, lane);
    default: return dq_tile<AT, UP, MOEB200_F32>(d, g, R, nkb, part, row, c0, sarea, ar, rw, rr, status, lane);
  }
}

// Waits (bounded, no status) for the last min(issued, depth) completions of a ring's full barriers:
// the issuing warp must not exit with its copies still landing.
__device__ __forceinline__ void drain(uint64_t* full, uint32_t issued, int depth) {
  const uint32_t dd = (uint32_t)depth;
  for (uint32_t q = issued > dd ? issued - dd : 0; q < issued; ++q) mbar_wait(&full[q % dd], (q / dd) & 1u, nullptr);
}

template <typename AT, bool UP>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const GemvParams p, const TcGeo g, const __grid_constant__ TcMaps tm) {
  constexpr int NA = UP ? 2 : 1;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - smem_u32(smem_raw));
  Rings R;
  R.a = sbase + g.a_off;
  R.b = sbase + g.b_off;
  R.r = sbase + g.r_off;
  R.s = sbase + g.s_off;
  R.d = sbase + g.d_off;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sgen + g.bar_off);
  R.afull = bars;
  R.aempty = R.afull + g.a_st;
  R.bfull = R.aempty + g.a_st;
  R.bempty = R.bfull + g.b_st;
  R.rfull = R.bempty + g.b_st;
  R.rempty = R.rfull + g.r_st;
  R.sfull = R.rempty + g.r_st;
  R.sempty = R.sfull + 2;
  R.accf = R.sempty + 2;
  R.acce = R.accf + 2;
  R.done = R.acce + 2;
  R.tmem_slot = reinterpret_cast<uint32_t*>(R.done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < g.a_st; ++s) {
      mbar_init(&R.afull[s], kDqWarps);
      mbar_init(&R.aempty[s], 1);
    }
    for (int s = 0; s < g.b_st; ++s) {
      mbar_init(&R.bfull[s], 1);
      mbar_init(&R.bempty[s], 1);
    }
    for (int s = 0; s < g.r_st; ++s) {
      mbar_init(&R.rfull[s], 1);
      mbar_init(&R.rempty[s], kDqWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&R.sfull[b], 1);
      mbar_init(&R.sempty[b], kDqWarps);
      mbar_init(&R.accf[b], 1);
      mbar_init(&R.acce[b], 4);
    }
    mbar_init(R.done, 1);
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(R.tmem_slot)),
                 "n"(UP ? 512 : 256));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *R.tmem_slot;
  constexpr int BUF_COLS = UP ? 256 : 128;  // one accumulator buffer (up: gate | up)

  const int n_items = *p.n_items;
  const int rb_per_item = (UP ? p.I : p.H) / BM;
  const int n_tiles = n_items * rb_per_item;
  const int nkb = (UP ? p.H : p.I) / BK;
  bool ok = true;

  if (warp < kDqWarps) {
    // ---------------- dequantisers ----------------
    const int tid = threadIdx.x;
    const int part = UP ? tid >> 8 : 0;
    const int row = UP ? (tid >> 1) & 127 : tid >> 2;
    const int c0 = UP ? (tid & 1) * 4 : (tid & 3) * 2;
    Ring ar, rw, rr;
    uint32_t sj = 0;
    for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
      TcTile d;
      tc_describe<UP>(p, tile, rb_per_item, d);
      const bool isint = is_int_w(d.wtype);
      uint32_t sarea = 0;
      if (isint) {
        const int par = sj & 1;
        if (!mbar_wait(&R.sfull[par], (sj >> 1) & 1u, p.status)) { ok = false; break; }
        sarea = R.s + par * g.s_bytes;
      }
      ok = dq_dispatch<AT, UP>(d, g, R, nkb, part, row, c0, sarea, ar, rw, rr, p.status, lane);
      if (isint) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&R.sempty[sj & 1]);
        ++sj;
      }
    }
  } else if (warp == kTmaWarp) {
    // ---------------- TMA producer: raw weight units and scale rows ----------------
    Ring rw;
    uint32_t issued = 0, sj = 0, jn = 0;
    const uint64_t tmap0 = reinterpret_cast<uint64_t>(p.tmap_ws) + (uint64_t)blockIdx.x * kTmapSlots * 128;
    for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
      TcTile d;
      tc_describe<UP>(p, tile, rb_per_item, d);
      // a tensor-map slot is reused after tmap_ring = r_st + 1 tiles: at most r_st units (so at most
      // r_st tiles) can still be landing, so the copies through the slot have completed
      const uint64_t gdesc = tmap0 + (uint64_t)(jn % (uint32_t)g.tmap_ring) * 128;
      ++jn;
      retarget_tmap(tm.w[d.slot], R.d, gdesc, d.q, lane);
      if (is_int_w(d.wtype)) {
        const int par = sj & 1;
        if (sj >= 2 && !mbar_wait(&R.sempty[par], ((sj >> 1) - 1) & 1u, p.status)) { ok = false; break; }
        if (lane == 0) {
          const uint32_t blk = (uint32_t)(BM * d.sstride);
          uint8_t* sa = sgen + g.s_off + par * g.s_bytes;
          mbar_arrive_expect_tx(&R.sfull[par], NA * blk);
          bulk_g2s(sa, d.s + (int64_t)d.r0 * d.sstride, blk, &R.sfull[par]);
          if (UP) bulk_g2s(sa + blk, d.s + (int64_t)(p.I + d.r0) * d.sstride, blk, &R.sfull[par]);
        }
        ++sj;
      }
      for (int u = 0; u < d.units; ++u) {
        if (!mbar_wait(&R.rempty[rw.slot], rw.phase ^ 1u, p.status)) { ok = false; break; }
        if (lane == 0) {
          const uint32_t dst = R.r + rw.slot * (NA * kTileBytes);
          mbar_arrive_expect_tx(&R.rfull[rw.slot], NA * kTileBytes);
          tma2d(dst, gdesc, u * 128, d.r0, &R.rfull[rw.slot]);
          if (UP) tma2d(dst + kTileBytes, gdesc, u * 128, p.I + d.r0, &R.rfull[rw.slot]);
        }
        __syncwarp();
        rw.next(g.r_st);
        ++issued;
      }
    }
    if (lane == 0) {
      drain(R.rfull, issued, g.r_st);
      if (sj) drain(R.sfull, sj, 2);
    }
    __syncwarp();
  } else if (warp == kLoadWarp) {
    // ---------------- B ring: token rows (up, cp.async gather) or h rows (down, TMA) ----------------
    Ring bw, bs;
    uint32_t issued = 0;
    int pending = 0;
    for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
      TcTile d;
      tc_describe<UP>(p, tile, rb_per_item, d);
      if constexpr (UP) {
        // per-lane rows: lane handles rows lane, lane+32, ... of the N-row B tile
        const AT* rowp[NMAX / 32];
#pragma unroll
        for (int i = 0; i < NMAX / 32; ++i) {
          const int j = lane + 32 * i;
          rowp[i] = static_cast<const AT*>(p.x);  // zero-filled (src size 0)
          if (j < d.ntok) rowp[i] += (int64_t)(p.pos[d.start + j] / p.k) * p.H;
        }
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&R.bempty[bw.slot], bw.phase ^ 1u, p.status)) { ok = false; break; }
          const uint32_t btile = R.b + bw.slot * kTileBytes;
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
          bw.next(g.b_st);
          if (++pending > g.lag) {
            cp_async_wait_n(g.lag);
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) mbar_arrive(&R.bfull[bs.slot]);
            bs.next(g.b_st);
            --pending;
          }
        }
      } else {
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&R.bempty[bw.slot], bw.phase ^ 1u, p.status)) { ok = false; break; }
          if (lane == 0) {
            mbar_arrive_expect_tx(&R.bfull[bw.slot], kTileBytes);
            tma2d(R.b + bw.slot * kTileBytes, reinterpret_cast<uint64_t>(&tm.h), kb * BK, d.start, &R.bfull[bw.slot]);
          }
          __syncwarp();
          bw.next(g.b_st);
          ++issued;
        }
      }
    }
    if constexpr (UP) {
      cp_async_wait<0>();
      fence_proxy_async();
      __syncwarp();
      if (lane == 0)
        for (; pending > 0; --pending) {
          mbar_arrive(&R.bfull[bs.slot]);
          bs.next(g.b_st);
        }
    } else {
      if (lane == 0) drain(R.bfull, issued, g.b_st);
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer (one thread) ----------------
    if (lane == 0) {
      Ring ar, br;
      uint32_t tcount = 0;
      for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x, ++tcount) {
        TcTile d;
        tc_describe<UP>(p, tile, rb_per_item, d);
        const int buf = tcount & 1;
        if (!mbar_wait(&R.acce[buf], ((tcount >> 1) & 1u) ^ 1u, p.status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t idesc = idesc_f16(std::is_same<AT, __nv_bfloat16>::value, d.n);
        const uint32_t d0 = tmem + buf * BUF_COLS;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&R.afull[ar.slot], ar.phase, p.status) || !mbar_wait(&R.bfull[br.slot], br.phase, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t astage = R.a + ar.slot * (NA * kTileBytes);
          const uint32_t btile = R.b + br.slot * kTileBytes;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t bdesc = sw128_desc(btile + kk * 32);
            const uint32_t accum = (kb > 0 || kk > 0) ? 1u : 0u;
            tc_mma(d0, sw128_desc(astage + kk * 32), bdesc, idesc, accum);
            if (UP) tc_mma(d0 + NMAX, sw128_desc(astage + kTileBytes + kk * 32), bdesc, idesc, accum);
          }
          tc_commit(&R.aempty[ar.slot]);
          tc_commit(&R.bempty[br.slot]);
          ar.next(g.a_st);
          br.next(g.b_st);
        }
        if (!ok) break;
        tc_commit(&R.accf[buf]);
      }
      tc_commit(R.done);
      mbar_wait(R.done, 0, p.status);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue warps (kEpiWarp0 .. kEpiWarp0 + 3) ----------------
    const int q = warp - kEpiWarp0;  // TMEM lane quarter
    const int r_local = q * 32 + lane;
    if (UP && p.zero_acc) {  // the down phase reduces into acc: clear it while the first tile runs
      const int64_t n4 = (int64_t)p.T * p.H / 4;
      float4* a4 = reinterpret_cast<float4*>(p.acc);
      for (int64_t i = (int64_t)blockIdx.x * 128 + q * 32 + lane; i < n4; i += (int64_t)gridDim.x * 128)
        a4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    uint32_t tcount = 0;
    for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x, ++tcount) {
      TcTile d;
      tc_describe<UP>(p, tile, rb_per_item, d);
      const int buf = tcount & 1;
      // down: this lane's tokens (pairs lane + 32 i) as acc row offsets and router weights
      int64_t toff[NMAX / 32];
      float wj[NMAX / 32];
      if constexpr (!UP) {
#pragma unroll
        for (int i = 0; i < NMAX / 32; ++i) {
          const int j = lane + 32 * i;
          toff[i] = 0;
          wj[i] = 0.f;
          if (j < d.ntok) {
            const int pos = p.pos[d.start + j];
            toff[i] = (int64_t)(pos / p.k) * p.H;
            wj[i] = p.wflat[pos];
          }
        }
      }
      if (!mbar_wait(&R.accf[buf], (tcount >> 1) & 1u, p.status)) { ok = false; break; }
      tc_fence_after();
      const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + buf * BUF_COLS;
      const int row = d.r0 + r_local;
#pragma unroll
      for (int j0 = 0; j0 < NMAX; j0 += 16) {
        if (j0 < d.n) {
          uint32_t a[16];
          tmem_ld16(tb + j0, a);
          if constexpr (UP) {
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
              const int64_t t = __shfl_sync(0xffffffffu, toff[j >> 5], j & 31);
              const float w = __shfl_sync(0xffffffffu, wj[j >> 5], j & 31);
              if (j < d.ntok) red_add_f32(p.acc + t + row, w * __uint_as_float(a[jj]));
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&R.acce[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(UP ? 512 : 256));
  }
}

// Ring depths for a phase: the first candidate whose shared memory fits one CTA.
bool plan_geo(bool up, uint32_t s_bytes, TcGeo& g, int& smem) {
  static const int cand_up[][3] = {{2, 4, 2}, {2, 3, 2}, {2, 2, 2}, {2, 2, 1}};
  static const int cand_dn[][3] = {{4, 4, 5}, {3, 4, 4}, {3, 3, 3}, {2, 2, 2}, {2, 2, 1}};
  const int na = up ? 2 : 1;
  const int nc = up ? 4 : 5;
  for (int i = 0; i < nc; ++i) {
    const int* c = up ? cand_up[i] : cand_dn[i];
    g.a_st = c[0];
    g.b_st = c[1];
    g.r_st = c[2];
    g.a_off = 0;
    g.b_off = g.a_off + (uint32_t)(g.a_st * na * kTileBytes);
    g.r_off = g.b_off + (uint32_t)(g.b_st * kTileBytes);
    g.s_off = g.r_off + (uint32_t)(g.r_st * na * kTileBytes);
    g.s_bytes = s_bytes;
    g.d_off = g.s_off + 2 * s_bytes;
    g.bar_off = g.d_off + 128;
    const uint32_t nbars = 2 * (g.a_st + g.b_st + g.r_st) + 9;
    smem = (int)(g.bar_off + nbars * 8 + 16 + 1024);
    if (smem <= kMaxSmem) {
      // the loader signals stage kb after issuing kb + lag, which needs stage kb + lag - b_st free:
      // lag = b_st - 2 leaves the MMA one stage of slack
      g.lag = std::max(0, g.b_st - 2);
      g.tmap_ring = g.r_st + 1;
      return true;
    }
  }
  return false;
}

template <typename AT, bool UP>
cudaError_t launch_tc_t(const GemvParams& p, const TcGeo& g, const TcMaps& tm, int smem, int grid, cudaStream_t s) {
  auto kern = gemm_tc_kernel<AT, UP>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, kThreads, smem, s>>>(p, g, tm);
  return cudaGetLastError();
}

cudaError_t launch_gemm_phase(const GemvParams& p, const moeb200_layout* lays, int nlay, int act, int n_pairs,
                              bool up, int grid, cudaStream_t s) {
  const int K = up ? p.H : p.I;
  const int na = up ? 2 : 1;
  uint32_t sst = 0;
  for (int i = 0; i < nlay; ++i) {
    const int wt = lays[i].wtype;
    if (wt == MOEB200_I4 || wt == MOEB200_I8) sst = std::max<uint32_t>(sst, (uint32_t)(K / (up ? lays[i].gs_up : lays[i].gs_dn) * 2));
  }
  const uint32_t s_bytes = (uint32_t)((na * BM * sst + 127) / 128 * 128);
  TcGeo g{};
  int smem = 0;
  if (!plan_geo(up, s_bytes, g, smem)) return cudaErrorInvalidConfiguration;
  TcMaps tm{};
  for (int i = 0; i < nlay; ++i) {
    cudaError_t e = tma_weight_template(&tm.w[i], K * gemv_wbits(lays[i].wtype) / 8, up ? 2 * p.I : p.H, BM, p.tmap_ws);
    if (e != cudaSuccess) return e;
  }
  if (!up) {
    cudaError_t e = tma_rows16_map(&tm.h, p.h, p.I, std::max(n_pairs, 1), BM, act);
    if (e != cudaSuccess) return e;
  }
  if (act == MOEB200_BF16)
    return up ? launch_tc_t<__nv_bfloat16, true>(p, g, tm, smem, grid, s)
              : launch_tc_t<__nv_bfloat16, false>(p, g, tm, smem, grid, s);
  return up ? launch_tc_t<__half, true>(p, g, tm, smem, grid, s) : launch_tc_t<__half, false>(p, g, tm, smem, grid, s);
}

}  // namespace

cudaError_t launch_gemm_up(const GemvParams& p, const moeb200_layout* lays, int nlay, int act_type, int n_pairs,
                           int grid, cudaStream_t s) {
  return launch_gemm_phase(p, lays, nlay, act_type, n_pairs, true, grid, s);
}

cudaError_t launch_gemm_down(const GemvParams& p, const moeb200_layout* lays, int nlay, int act_type, int n_pairs,
                             int grid, cudaStream_t s) {
  return launch_gemm_phase(p, lays, nlay, act_type, n_pairs, false, grid, s);
}

}  // namespace moeb200
