// Warp-streamed grouped GEMV -- the small-batch decode path of the MoE layer.
//
// Replaces, for work items of at most 8 routed pairs, the same Triton grouped kernels as gemv.cu
// (moelab kernels.py `_grp4_up` 312-361, `_grp4_down` 363-396, `_grp8_*` 667-740, `_grpf_*`
// 398-451) with the same results:
//
//   up   : h[j, r]  = silu(gate_r . x_tok(j)) * (up_r . x_tok(j))       for each pair j of an item
//   down : acc[t, r] += w_j * (down_r . h[j])                            (fp32 reduction = combine)
//
// At decode batch sizes a layer streams a few MB of records per phase, ~100 KB per SM, so the
// phase time is set by how soon every SM has its bytes in flight. Plain loads cannot do that: the
// misses an SM can hold outstanding cap it near 11 GB/s at these latencies (measured: 1.6 TB/s for
// the whole chip with 128 KB of loads issued per SM). Here every warp streams its own weight rows
// through the copy engine into two 5 KB shared-memory slots of its own -- the next chunk always in
// flight while it multiplies the current one -- so each SM keeps up to 128 KB of records in flight
// with no producer warp or cross-warp hand-off. A chunk is 256 bytes of each of the warp's 16 rows,
// moved as 2-D TMA boxes of 128 bytes x 8 (gate/up) or 16 (down) rows from a tensor map of all
// memory above the expert table's tma_base (records lie on row multiples above it, so no map is
// built per record) -- four or two tensor loads per chunk plus one or two bulk copies of the tile's
// whole scale rows, where per-row 1-D copies took 32: the copy engine's per-request cost, not DRAM,
// bounded that version. The boxes land 128-byte swizzled, so the fragment reads of the warp's rows
// fall in different banks. A chunk's groups are multiplied in a fully unrolled sequence, and a CTA
// runs 16 warps when their slots fit beside the activation rows (8 else), so each scheduler has 4
// warps' independent dequantise-and-multiply chains to interleave.
//
// Fragment layout. A warp owns one 16-row mma.sync m16n8k16 tile: up = 8 gate rows (tile rows
// 0..7) and the matching 8 up rows (tile rows 8..15), so gate and up of one intermediate row land
// in the same lane and SwiGLU happens in registers; down = 16 consecutive output rows. K is walked
// in 64-column groups; in a group, lane (g, t) holds columns 16t..16t+15 of its rows g and g+8
// (int4: 8 bytes per row, int8: 16, 16-bit floats: 32), so every mma sums columns of one scale
// group: the exact integer products of the group are summed in fp32 and the group's partial is
// scaled once (as gemv.cu does). In a slot, byte b of box row r lies at
// (b / 128) * SS + r * 128 + (((b / 16) % 8) ^ (r % 8)) * 16 + b % 16, SS = 1 KB (8-row boxes) or 2 KB
// (16 rows); rows g and g + 8 share r % 8 = g. The item's activation rows (B fragments) are staged
// in shared memory with bulk copies, double-buffered across work units.
//
// Work. A CTA (one per SM) takes units = (item, row block, all K): its warps split the
// row block into 16-row tiles and, when a call has few items, K into ks parts (warp w: tile w / ks,
// part w % ks); the parts of a tile are added in part order through shared memory (the same sum on
// every run). The down kernel issues its first weight copies before it waits for the gate/up
// kernel (only h comes from it), so its first DRAM round trip overlaps the gate/up tail.
#include "gemv.cuh"
#include "tma.cuh"

namespace moeb200 {

namespace {

constexpr int kWsMaxWarps = 16;
constexpr int kWsMaxTok = 8;      // pairs of one item: one mma column block
constexpr int kWsSegBytes = 256;  // weight bytes of one row per chunk
constexpr int kWsWBytes = 16 * kWsSegBytes;  // the chunk's 16 rows: two 128-byte segments of swizzled boxes

enum WsKind : int { kWsI4 = 0, kWsI8 = 1, kWsF = 2 };

// Per kind: NG = 64-column groups of one chunk (256 weight bytes per row).
template <int KIND>
struct WsGeo;
template <>
struct WsGeo<kWsI4> {
  static constexpr int NG = 8;
};
template <>
struct WsGeo<kWsI8> {
  static constexpr int NG = 4;
};
template <>
struct WsGeo<kWsF> {
  static constexpr int NG = 2;
};

// A slot of a phase with K columns: the chunk's weight boxes, then the 16 rows' whole scale rows
// (16 * K / 64 * 2 bytes), rounded up to 1 KB so that every slot's boxes start on a 1024-byte
// boundary (the period of the 128-byte swizzle).
__host__ __device__ inline int ws_slot_bytes(int K) { return kWsWBytes + ((K / 2 + 1023) / 1024) * 1024; }

// Tensor maps of the weight fields, per precision slot and phase (0 gate/up, 1 down): uint8 [rows][row
// bytes] views of the memory above tma_base, boxes of 128 bytes x 8 (gate/up) or 16 (down) rows.
struct alignas(64) WsMaps {
  CUtensorMap m[4][2];
};

__device__ __forceinline__ int ws_kind(int wtype) {
  return wtype == MOEB200_I4 ? kWsI4 : wtype == MOEB200_I8 ? kWsI8 : kWsF;
}
__device__ __forceinline__ int ws_cc(int kind) {  // columns of one chunk
  return 64 * (kind == kWsI4 ? WsGeo<kWsI4>::NG : kind == kWsI8 ? WsGeo<kWsI8>::NG : WsGeo<kWsF>::NG);
}
__device__ __forceinline__ int ws_cc_log2(int kind) {  // log2 of ws_cc (512, 256, 128 columns)
  return kind == kWsI4 ? 9 : kind == kWsI8 ? 8 : 7;
}

// n / d for 0 <= n and d >= 1 without an integer division sequence on the units' critical path:
// for n < 2^22 the float quotient n * (1/d) (reciprocal correctly rounded) is within one of n / d, so
// one remainder check makes it exact; larger n take the integer division.
__device__ __forceinline__ int small_div(int n, int d, float inv) {
  if (n >= (1 << 22)) return n / d;
  int q = __float2int_rz(__int2float_rn(n) * inv);
  const int r = n - q * d;
  if (r < 0) --q;
  else if (r >= d) ++q;
  return q;
}

__device__ __forceinline__ uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ float half_lo(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFFu))); }
__device__ __forceinline__ float half_hi(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }

// One chunk (NG groups, unrolled) of the lane's rows g and g+8: ra / rb = shared address of the
// rows' first segment in the slot's boxes, ss = bytes between two segments of a row, sa / sb = the
// rows' scales of the chunk's first group, xs = shared address of the lane's token row at the
// chunk's first column plus 32t; xon = the lane's token exists.
template <typename AT, int KIND>
__device__ __forceinline__ void ws_chunk(uint32_t ra, uint32_t rb, uint32_t ss, uint32_t sa, uint32_t sb, uint32_t xs,
                                         bool xon, int g, int t, float (&tot)[4]) {
  using G = WsGeo<KIND>;
  if constexpr (KIND == kWsI4) {
    // the 8 groups' scales of both rows: 16 bytes per row
    const uint4 sg = lds128(sa), su = lds128(sb);
    const uint32_t sgw[4] = {sg.x, sg.y, sg.z, sg.w}, suw[4] = {su.x, su.y, su.z, su.w};
    // the lane's 8 bytes of group j: segment j / 4, 16-byte unit (2 (j % 4) + t / 2) ^ g
    uint32_t uo[4];
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) uo[jj] = ((uint32_t)((2 * jj + (t >> 1)) ^ g) << 4) + 8u * (t & 1);
#pragma unroll
    for (int j = 0; j < G::NG; ++j) {
      const uint32_t off = (uint32_t)(j >> 2) * ss + uo[j & 3];
      const uint2 wg = lds64(ra + off), wu = lds64(rb + off);
      uint4 X0 = make_uint4(0, 0, 0, 0), X1 = X0;
      if (xon) {
        X0 = lds128(xs + j * 128);
        X1 = lds128(xs + j * 128 + 16);
      }
      const uint32_t w0[2] = {wg.x, wg.y}, w1[2] = {wu.x, wu.y};
      const uint32_t xw[8] = {X0.x, X0.y, X0.z, X0.w, X1.x, X1.y, X1.z, X1.w};
      float d[4];
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        uint32_t p04[2], p15[2], p26[2], p37[2];
        Dq<AT>::int4x8(w0[m], p04[0], p15[0], p26[0], p37[0]);
        Dq<AT>::int4x8(w1[m], p04[1], p15[1], p26[1], p37[1]);
        const uint32_t x0 = xw[4 * m], x1 = xw[4 * m + 1], x2 = xw[4 * m + 2], x3 = xw[4 * m + 3];
        const uint32_t a0[4] = {p04[0], p04[1], p15[0], p15[1]};
        const uint32_t a1[4] = {p26[0], p26[1], p37[0], p37[1]};
        if (m == 0)
          MmaOp<AT>::first(d, a0, prmt(x0, x2, 0x5410), prmt(x0, x2, 0x7632));
        else
          MmaOp<AT>::run(d, a0, prmt(x0, x2, 0x5410), prmt(x0, x2, 0x7632));
        MmaOp<AT>::run(d, a1, prmt(x1, x3, 0x5410), prmt(x1, x3, 0x7632));
      }
      const float s0 = (j & 1) ? half_hi(sgw[j >> 1]) : half_lo(sgw[j >> 1]);
      const float s1 = (j & 1) ? half_hi(suw[j >> 1]) : half_lo(suw[j >> 1]);
      tot[0] = fmaf(s0, d[0], tot[0]);
      tot[1] = fmaf(s0, d[1], tot[1]);
      tot[2] = fmaf(s1, d[2], tot[2]);
      tot[3] = fmaf(s1, d[3], tot[3]);
    }
  } else if constexpr (KIND == kWsI8) {
    // the 4 groups' scales of both rows: 8 bytes per row
    const uint2 sg = lds64(sa), su = lds64(sb);
    const uint32_t sgw[2] = {sg.x, sg.y}, suw[2] = {su.x, su.y};
    // the lane's 16 bytes of group j: segment j / 2, 16-byte unit (4 (j % 2) + t) ^ g
    const uint32_t uo[2] = {(uint32_t)(t ^ g) << 4, (uint32_t)((4 + t) ^ g) << 4};
#pragma unroll
    for (int j = 0; j < G::NG; ++j) {
      const uint32_t off = (uint32_t)(j >> 1) * ss + uo[j & 1];
      const uint4 wg = lds128(ra + off), wu = lds128(rb + off);
      uint4 X0 = make_uint4(0, 0, 0, 0), X1 = X0;
      if (xon) {
        X0 = lds128(xs + j * 128);
        X1 = lds128(xs + j * 128 + 16);
      }
      const uint32_t w0[4] = {wg.x, wg.y, wg.z, wg.w}, w1[4] = {wu.x, wu.y, wu.z, wu.w};
      const uint32_t xw[8] = {X0.x, X0.y, X0.z, X0.w, X1.x, X1.y, X1.z, X1.w};
      float d[4];
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        uint32_t p01[2], p23[2];
        Dq<AT>::int8x4(w0[m], p01[0], p23[0]);
        Dq<AT>::int8x4(w1[m], p01[1], p23[1]);
        const uint32_t a[4] = {p01[0], p01[1], p23[0], p23[1]};
        if (m == 0)
          MmaOp<AT>::first(d, a, xw[2 * m], xw[2 * m + 1]);
        else
          MmaOp<AT>::run(d, a, xw[2 * m], xw[2 * m + 1]);
      }
      const float s0 = (j & 1) ? half_hi(sgw[j >> 1]) : half_lo(sgw[j >> 1]);
      const float s1 = (j & 1) ? half_hi(suw[j >> 1]) : half_lo(suw[j >> 1]);
      tot[0] = fmaf(s0, d[0], tot[0]);
      tot[1] = fmaf(s0, d[1], tot[1]);
      tot[2] = fmaf(s1, d[2], tot[2]);
      tot[3] = fmaf(s1, d[3], tot[3]);
    }
  } else {
    // the lane's 32 bytes of group j: segment j's 16-byte units 2t ^ g and (2t + 1) ^ g
    const uint32_t u0 = (uint32_t)((2 * t) ^ g) << 4, u1 = (uint32_t)((2 * t + 1) ^ g) << 4;
#pragma unroll
    for (int j = 0; j < G::NG; ++j) {
      const uint32_t so = (uint32_t)j * ss;
      const uint4 g0 = lds128(ra + so + u0), g1 = lds128(ra + so + u1);
      const uint4 v0 = lds128(rb + so + u0), v1 = lds128(rb + so + u1);
      uint4 X0 = make_uint4(0, 0, 0, 0), X1 = X0;
      if (xon) {
        X0 = lds128(xs + j * 128);
        X1 = lds128(xs + j * 128 + 16);
      }
      const uint32_t w0[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
      const uint32_t w1[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
      const uint32_t xw[8] = {X0.x, X0.y, X0.z, X0.w, X1.x, X1.y, X1.z, X1.w};
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const uint32_t a[4] = {w0[2 * m], w1[2 * m], w0[2 * m + 1], w1[2 * m + 1]};
        MmaOp<AT>::run(tot, a, xw[2 * m], xw[2 * m + 1]);
      }
    }
  }
}

// Geometry of one unit for one warp.
struct WsUnit {
  Item it;
  int kind;
  int r0;       // first row of the warp's tile (up: first gate row)
  int k0, kc;   // the warp's K part
  int nch;      // chunks in the part
  int row0;     // the phase's weight field's first row in the tensor maps' row coordinates
  bool live;    // a well-formed item in which the tile has rows
};


template <bool UP>
// ksl = log2 of the K parts (a power of two)
__device__ __forceinline__ WsUnit ws_unit(const GemvParams& p, const Item& it, int rb, int ksl, int nw, int warp) {
  WsUnit u;
  u.it = it;
  u.kind = ws_kind(p.lay[it.slot].wtype);
  const int K = UP ? p.H : p.I;
  const int rows = UP ? p.I : p.H;
  const int rpt = UP ? 8 : 16;
  u.r0 = (rb * (nw >> ksl) + (warp >> ksl)) * rpt;
  u.live = u.r0 < rows;
  u.kc = K >> ksl;
  u.k0 = (warp & ((1 << ksl) - 1)) * u.kc;
  u.nch = u.kc >> ws_cc_log2(u.kind);
  const int64_t rowb = (int64_t)K * (u.kind == kWsI4 ? 4 : u.kind == kWsI8 ? 8 : 16) / 8;
  // records lie on 4096-byte multiples above tma_base and the row pitches divide 4096 and the field
  // offsets, so -1 means a record the runtime did not place
  u.row0 = row_map_first(UP ? it.p_guq : it.p_dnq, p.tma_base, rowb, UP ? 2 * p.I : p.H);
  return u;
}

// The warp issues chunk c of its unit into its slot: lanes 0..3 (gate/up: 128-byte segment k of the
// 8 gate rows and of the 8 up rows) or 0..1 (down: segment k of the 16 rows) one TMA box each; the
// next lanes one bulk copy each of the tile's whole scale rows (integer records).
template <bool UP>
__device__ __forceinline__ void ws_issue(const GemvParams& p, const WsMaps& tm, const WsUnit& u, int c, uint8_t* slot,
                                         uint64_t* bar, int lane) {
  const int K = UP ? p.H : p.I;
  const int kind = u.kind;
  const int col0 = u.k0 + c * ws_cc(kind);
  const int wbits = kind == kWsI4 ? 4 : kind == kWsI8 ? 8 : 16;
  const uint32_t srow = kind != kWsF ? (uint32_t)(K / 64) * 2u : 0u;
  if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)kWsWBytes + 16u * srow);
  __syncwarp();
  const uint64_t map = reinterpret_cast<uint64_t>(&tm.m[u.it.slot][UP ? 0 : 1]);
  const uint32_t w = smem_u32(slot);
  const int x0 = col0 * wbits / 8;  // the chunk's first byte of a row
  const uint8_t* sc = reinterpret_cast<const uint8_t*>(UP ? u.it.p_gus : u.it.p_dns);
  if (UP) {
    if (lane < 4) {
      const int k = lane & 1, half = lane >> 1;  // half 0: gate rows, 1: up rows
      tma2d(w + 2048u * half + 1024u * k, map, x0 + 128 * k, u.row0 + half * p.I + u.r0, bar);
    } else if (lane < 6 && srow) {
      const int half = lane - 4;
      bulk_g2s(slot + kWsWBytes + 8u * srow * half, sc + (int64_t)(half * p.I + u.r0) * srow, 8u * srow, bar);
    }
  } else {
    if (lane < 2) {
      tma2d(w + 2048u * lane, map, x0 + 128 * lane, u.row0 + u.r0, bar);
    } else if (lane == 2 && srow) {
      bulk_g2s(slot + kWsWBytes, sc + (int64_t)u.r0 * srow, 16u * srow, bar);
    }
  }
}

// One phase, NW warps. Shared memory (from a 1024-byte boundary): weight slots [NW][2], activation
// rows [2][xrows][K + 8] (16-bit), part sums [NW * 32] float4, mbarriers: 2 activation buffers, 2 per
// warp.
template <typename AT, bool UP, int NW>
__global__ void __launch_bounds__(32 * NW, 1) ws_kernel(const GemvParams p, const __grid_constant__ WsMaps tm, int ks,
                                                        int xrows) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int K = UP ? p.H : p.I;
  const int xstride = K * 2 + 16;  // odd multiple of 16 bytes: the token rows fall in different banks
  const int slot_bytes = ws_slot_bytes(K);
  uint8_t* slots = smem;
  uint8_t* xbuf = smem + NW * 2 * slot_bytes;
  float4* part = reinterpret_cast<float4*>(xbuf + 2 * xrows * xstride);
  uint64_t* xfull = reinterpret_cast<uint64_t*>(part + 32 * NW);
  uint64_t* wfull = xfull + 2;  // [warp][2]
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2 + 2 * NW; ++i) mbar_init(&xfull[i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  uint8_t* myslot[2] = {slots + (warp * 2) * slot_bytes, slots + (warp * 2 + 1) * slot_bytes};

  const int rows = UP ? p.I : p.H;
  const int ksl = __ffs(ks) - 1;  // the K parts are a power of two
  const int rb_rows = (UP ? 8 : 16) * (NW >> ksl);
  const int upi = (rows + rb_rows - 1) / rb_rows;  // units per item
  // reciprocals for the per-unit quotients (small_div)
  const float inv_upi = __frcp_rn((float)upi), inv_k = __frcp_rn((float)p.k);

  // the warp's chunk stream: units cu = blockIdx.x, +gridDim.x, ...; chunks of the warp's K part
  int n_items = 0;
  uint32_t n_issued = 0, n_done = 0;
  int icu = blockIdx.x, ic = 0;  // next chunk to issue
  WsUnit iu{};
  bool ivalid = false;
  // a unit the warp takes part in; an item outside the kernel's limits (never written by the
  // dispatch) is flagged and its unit skipped by the warp's issue and compute streams alike
  auto load_unit = [&](int cu, WsUnit& u) -> bool {
    u.live = false;
    if (cu >= n_items * upi) return false;
    const int item = small_div(cu, upi, inv_upi);
    const Item it = p.items[item];
    if (it.ntok < 1 || it.ntok > xrows || it.slot < 0 || it.slot > 3) {
      if (lane == 0) atomicExch(p.status, kDevBadIndex);
      return true;
    }
    u = ws_unit<UP>(p, it, cu - item * upi, ksl, NW, warp);
    if (u.live && u.row0 < 0) {  // a record off the tensor maps' rows: flagged, its unit skipped
      if (lane == 0) atomicExch(p.status, kDevBadIndex);
      u.live = false;
    }
    return true;
  };
  // issue the next chunk of the stream (skipping units where the warp has no rows)
  auto issue_next = [&]() {
    while (ivalid && (!iu.live || ic >= iu.nch)) {
      icu += gridDim.x;
      ic = 0;
      ivalid = load_unit(icu, iu);
    }
    if (!ivalid) return;
    ws_issue<UP>(p, tm, iu, ic, myslot[n_issued & 1], &wfull[warp * 2 + (n_issued & 1)], lane);
    ++n_issued;
    ++ic;
  };

  // down: the items were written before the gate/up kernel started (it waited for their writer
  // before letting this kernel launch); the first weight copies go out before the wait for h
  if (!UP) {
    n_items = *p.n_items;
    ivalid = load_unit(icu, iu);
    issue_next();
  }
  chain_wait();
  chain_release();
  if (UP) {
    n_items = *p.n_items;
    ivalid = load_unit(icu, iu);
    issue_next();
  }
  if (UP && p.zero_acc) {  // the down phase reduces into acc; clear it first (grid-stride)
    const int64_t n = (int64_t)p.T * p.H;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
      p.acc[i] = 0.f;
  }

  // activation rows of unit ordinal n into buffer n & 1 (thread 0)
  auto stage = [&](int cu, uint32_t n) {
    const Item it = p.items[small_div(cu, upi, inv_upi)];
    uint64_t* bar = &xfull[n & 1];
    if (it.ntok < 1 || it.ntok > xrows) {  // flagged by load_unit; complete the phase empty
      mbar_arrive_expect_tx(bar, 0);
      return;
    }
    const uint32_t rowb = (uint32_t)K * 2;
    // the buffer's last readers (generic proxy) are ordered before these copies (async proxy)
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_arrive_expect_tx(bar, rowb * it.ntok);
    uint8_t* dst = xbuf + (n & 1) * xrows * xstride;
    for (int j = 0; j < it.ntok; ++j) {
      const uint8_t* src = UP ? static_cast<const uint8_t*>(p.x) + (int64_t)small_div(p.pos[it.start + j], p.k, inv_k) * rowb
                              : static_cast<const uint8_t*>(p.h) + (int64_t)(it.start + j) * rowb;
      bulk_g2s(dst + j * xstride, src, rowb, bar);
    }
  };
  const int n_cu = n_items * upi;
  if (threadIdx.x == 0 && (int)blockIdx.x < n_cu) stage(blockIdx.x, 0);

  bool ok = true;
  uint32_t n = 0;  // unit ordinal of this CTA
  for (int cu = blockIdx.x; cu < n_cu; cu += gridDim.x, ++n) {
    // the buffer of the next unit was last read by unit n - 1, which every warp has finished
    if (threadIdx.x == 0 && cu + (int)gridDim.x < n_cu) stage(cu + gridDim.x, n + 1);
    WsUnit u;
    load_unit(cu, u);
    const bool valid = u.live;
    float tot[4] = {0.f, 0.f, 0.f, 0.f};
    const bool xon = valid && g < u.it.ntok;
    const bool xready = mbar_wait(&xfull[n & 1], (n >> 1) & 1, p.status);
    ok = ok && xready;
    if (valid) {
      const uint32_t xs = smem_u32(xbuf) + (n & 1) * xrows * xstride + (uint32_t)(g * xstride) +
                          (uint32_t)(u.k0 * 2) + 32u * t;
      const int cc = ws_cc(u.kind);
      for (int c = 0; c < u.nch; ++c) {
        issue_next();  // the next chunk goes out before this one is multiplied
        const uint32_t sl = n_done & 1;
        const bool landed = mbar_wait(&wfull[warp * 2 + sl], (n_done >> 1) & 1, p.status);
        ++n_done;
        ok = ok && landed;
        if (landed && xready) {
          const uint32_t wsl = smem_u32(myslot[sl]);
          const uint32_t xc = xs + (uint32_t)(c * cc * 2);
          // rows g and g+8: gate/up = row g of the gate boxes and of the up boxes (8 rows, segments
          // 1 KB apart); down = rows g and g+8 of the 16-row boxes (segments 2 KB apart)
          const uint32_t ra = wsl + (uint32_t)g * 128u;
          const uint32_t rb = UP ? wsl + 2048u + (uint32_t)g * 128u : wsl + (uint32_t)(g + 8) * 128u;
          const uint32_t ss = UP ? 1024u : 2048u;
          // the rows' scales of the chunk's first group (whole scale rows follow the boxes)
          const uint32_t srow = (uint32_t)(K / 64) * 2u;
          const uint32_t g0 = (uint32_t)((u.k0 + c * cc) / 64) * 2u;
          const uint32_t sa = wsl + kWsWBytes + (uint32_t)g * srow + g0;
          const uint32_t sb = wsl + kWsWBytes + (uint32_t)(g + 8) * srow + g0;
          if (u.kind == kWsI4) ws_chunk<AT, kWsI4>(ra, rb, ss, sa, sb, xc, xon, g, t, tot);
          else if (u.kind == kWsI8) ws_chunk<AT, kWsI8>(ra, rb, ss, sa, sb, xc, xon, g, t, tot);
          else ws_chunk<AT, kWsF>(ra, rb, ss, sa, sb, xc, xon, g, t, tot);
        }
        // every lane is done with the slot before the copy that reuses it is issued
        __syncwarp();
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      }
    }
    // add the K parts of each tile in part order
    if (ks > 1) {
      part[threadIdx.x] = make_float4(tot[0], tot[1], tot[2], tot[3]);
      __syncthreads();
      if ((warp & (ks - 1)) == 0) {
        for (int q = 1; q < ks; ++q) {
          const float4 v = part[threadIdx.x + 32 * q];
          tot[0] += v.x;
          tot[1] += v.y;
          tot[2] += v.z;
          tot[3] += v.w;
        }
      }
    }
    if (valid && (warp & (ks - 1)) == 0 && ok) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int tk = 2 * t + e;
        if (tk >= u.it.ntok) continue;
        const int j = u.it.start + tk;
        if (UP) {
          static_cast<AT*>(p.h)[(int64_t)j * p.I + u.r0 + g] = from_f32<AT>(silu_mul(tot[e], tot[2 + e]));
        } else {
          const int pos = p.pos[j];
          float* arow = p.acc + (int64_t)small_div(pos, p.k, inv_k) * p.H + u.r0;
          const float wv = p.wflat[pos];
          red_add_f32(arow + g, wv * tot[e]);
          red_add_f32(arow + 8 + g, wv * tot[2 + e]);
        }
      }
    }
    __syncthreads();  // part sums and the activation buffer of this unit are reused two units on
  }
  // no copy may be in flight when the CTA exits (after a failed wait some may still be landing)
  while (n_done < n_issued) {
    mbar_wait(&wfull[warp * 2 + (n_done & 1)], (n_done >> 1) & 1, nullptr);
    ++n_done;
  }
}

size_t ws_smem(int K, int nw, int xrows) {
  return 1024 /* alignment of the slots */ + (size_t)nw * 2 * ws_slot_bytes(K) + (size_t)2 * xrows * (K * 2 + 16) +
         (size_t)nw * 32 * 16 + (2 + 2 * nw) * 8;
}

// Warps of a CTA: 16 when their slots fit beside the activation rows, else 8.
int ws_warps(int K, int xrows) { return ws_smem(K, 16, xrows) <= 227 * 1024 ? 16 : 8; }

template <typename AT, bool UP, int NW>
cudaError_t ws_launch_nw(const GemvParams& p, const WsMaps& tm, int ks, int xrows, int grid, cudaStream_t s) {
  const int K = UP ? p.H : p.I;
  const size_t smem = ws_smem(K, NW, xrows);
  cudaError_t e = cudaFuncSetAttribute(ws_kernel<AT, UP, NW>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return launch_chained(ws_kernel<AT, UP, NW>, dim3(grid), dim3(32 * NW), smem, s, p, tm, ks, xrows);
}

template <typename AT, bool UP>
cudaError_t ws_launch(const GemvParams& p, const WsMaps& tm, int nw, int ks, int xrows, int grid, cudaStream_t s) {
  return nw == 16 ? ws_launch_nw<AT, UP, 16>(p, tm, ks, xrows, grid, s)
                  : ws_launch_nw<AT, UP, 8>(p, tm, ks, xrows, grid, s);
}

// K parts of a phase: the fewest (1, 2, 4, ...) whose units give every SM work, keeping every part
// a multiple of 512 columns (whole chunks of every kind).
int ws_choose_ks(int max_items, int rows, int K, int rpt, int nw, int sms) {
  int ks = 1;
  while (ks < nw) {
    const int rb_rows = rpt * (nw / ks);
    const int64_t units = (int64_t)max_items * ((rows + rb_rows - 1) / rb_rows);
    if (units >= sms) break;
    if (K % (2 * ks * 512)) break;
    ks *= 2;
  }
  return ks;
}

}  // namespace

bool ws_supported(const moeb200_layout* lays, int nlay, int act_type, int H, int I, int max_item_pairs) {
  if (act_type != MOEB200_F16 && act_type != MOEB200_BF16) return false;
  if (max_item_pairs > kWsMaxTok) return false;
  if (H % 512 || I % 512) return false;  // K parts of whole chunks of every kind
  for (int i = 0; i < nlay; ++i) {
    const moeb200_layout& L = lays[i];
    const bool isint = L.wtype == MOEB200_I4 || L.wtype == MOEB200_I8;
    if (isint) {
      if (L.gs_up != 64 || L.gs_dn != 64) return false;
    } else if (L.wtype != act_type) {
      return false;  // float records are read as the activation type
    }
    // scale fields 16-byte aligned inside the record (bulk copies)
    if (isint && (L.off_gu_s % 16 || L.off_dn_s % 16)) return false;
    // tensor-map rows: records lie on 4096-byte multiples above the maps' base, so the row pitches
    // must divide 4096 and the weight field offsets
    const int bits = gemv_wbits(L.wtype);
    const int rb_up = H * bits / 8, rb_dn = I * bits / 8;
    if (4096 % rb_up || 4096 % rb_dn || L.off_gu_q % rb_up || L.off_dn_q % rb_dn) return false;
  }
  return ws_smem(std::max(H, I), 8, kWsMaxTok) <= 227 * 1024;
}

cudaError_t launch_ws_phases(GemvParams& p, const moeb200_layout* lays, int nlay, int act_type, int max_items,
                             cudaStream_t s) {
  const int sms = num_sms_cached();
  const int xrows = std::min(kWsMaxTok, p.T);  // an item holds at most this many pairs
  const int nw_up = ws_warps(p.H, xrows), nw_dn = ws_warps(p.I, xrows);
  const int ks_up = ws_choose_ks(max_items, p.I, p.H, 8, nw_up, sms);
  const int ks_dn = ws_choose_ks(max_items, p.H, p.I, 16, nw_dn, sms);
  const int rb_up = 8 * (nw_up / ks_up), rb_dn = 16 * (nw_dn / ks_dn);
  const int64_t cu_up = (int64_t)max_items * ((p.I + rb_up - 1) / rb_up);
  const int64_t cu_dn = (int64_t)max_items * ((p.H + rb_dn - 1) / rb_dn);
  const int grid_up = (int)std::max<int64_t>(1, std::min<int64_t>(sms, cu_up));
  const int grid_dn = (int)std::max<int64_t>(1, std::min<int64_t>(sms, cu_dn));
  p.ksplit_up = p.ksplit_dn = 1;
  if (p.tma_base == 0 || p.tma_base % 4096) return cudaErrorInvalidValue;
  WsMaps tm{};
  for (int i = 0; i < nlay && i < 4; ++i) {
    const int bits = gemv_wbits(lays[i].wtype);
    const int rb_up = p.H * bits / 8, rb_dn = p.I * bits / 8;
    cudaError_t e = tma_rows2d_map(&tm.m[i][0], (uint64_t)p.tma_base, rb_up, row_map_rows(rb_up), 8);
    if (e != cudaSuccess) return e;
    e = tma_rows2d_map(&tm.m[i][1], (uint64_t)p.tma_base, rb_dn, row_map_rows(rb_dn), 16);
    if (e != cudaSuccess) return e;
  }
  cudaError_t e = trace_mark(0, s);
  if (e != cudaSuccess) return e;
  e = act_type == MOEB200_BF16 ? ws_launch<__nv_bfloat16, true>(p, tm, nw_up, ks_up, xrows, grid_up, s)
                               : ws_launch<__half, true>(p, tm, nw_up, ks_up, xrows, grid_up, s);
  if (e != cudaSuccess) return e;
  e = trace_mark(1, s);
  if (e != cudaSuccess) return e;
  e = act_type == MOEB200_BF16 ? ws_launch<__nv_bfloat16, false>(p, tm, nw_dn, ks_dn, xrows, grid_dn, s)
                               : ws_launch<__half, false>(p, tm, nw_dn, ks_dn, xrows, grid_dn, s);
  if (e != cudaSuccess) return e;
  return trace_mark(2, s);
}

}  // namespace moeb200
