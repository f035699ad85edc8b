// Grouped expert GEMV -- the decode path of the MoE layer on B200.
//
// Replaces the Triton grouped kernels of moelab (kernels.py `_grp4_up` 312-361, `_grp4_down`
// 363-396, `_grp8_up/_grp8_down` 667-740, `_grpf_up/_grpf_down` 398-451) with one warp-level
// pipeline per phase:
//
//   up   : h[j, r]  = silu(gate_r . x_tok(j)) * (up_r . x_tok(j))      for each pair j of an item
//   down : acc[t, r] += w_j * (down_r . h[j])                           (fp32 reduction = combine)
//
// Work is split into warp tiles (item, 32 weight rows, K split): the up phase pairs 16 gate rows
// with the 16 matching up rows so SwiGLU happens in registers; the down phase takes 32 consecutive
// rows. Each warp streams its rows through its own ring of shared-memory stages filled by 1-D bulk
// TMA copies (one 256-byte row segment per lane per stage; padded row strides keep the fragment
// reads bank-conflict free), dequantises int4/int8 in registers straight into tensor-core A
// fragments and multiplies them with the activations of up to 8*NB tokens on mma.sync m16n8k16
// (fp32 accumulators, two independent accumulator sets per chunk so consecutive MMAs do not wait on
// each other). The fp16 group scale multiplies the fp32 partial of each chunk (a chunk never
// straddles a group), so weights are never rounded. The activation operand of the next chunk is
// loaded while the current one is multiplied.
//
// Small batches split K across warps: the up phase then adds fp32 partial pre-activations into
// pre[j, 0:2I] (gate | up); the warp whose split of a tile arrives last (a per-tile counter) forms
// h = silu(gate) * up for the tile's 16 rows, so the down phase always reads h.
#include <type_traits>

#include "gemv.cuh"

namespace moeb200 {

namespace {

enum Kind : int32_t {
  kI4w2 = 0, kI4w1, kI8w4, kI8w2, kI8w1, kF16w4, kF16w2, kF16w1, kBF16w4, kBF16w2, kBF16w1, kF32w2, kF32w1,
  kBadKind
};

__device__ __forceinline__ int wbits_of(int wtype) {
  return wtype == MOEB200_I4 ? 4 : wtype == MOEB200_I8 ? 8 : wtype == MOEB200_F32 ? 32 : 16;
}

__device__ __forceinline__ int kind_of(int wtype, int K, int gs) {
  switch (wtype) {
    case MOEB200_I4:
      if (gs % 64 == 0 && K % 64 == 0) return kI4w2;
      if (gs % 32 == 0 && K % 32 == 0) return kI4w1;
      return kBadKind;
    case MOEB200_I8:
      if (gs % 64 == 0 && K % 64 == 0) return kI8w4;
      if (gs % 32 == 0 && K % 32 == 0) return kI8w2;
      if (gs % 16 == 0 && K % 16 == 0) return kI8w1;
      return kBadKind;
    case MOEB200_F16:
      return K % 64 == 0 ? kF16w4 : K % 32 == 0 ? kF16w2 : K % 16 == 0 ? kF16w1 : kBadKind;
    case MOEB200_BF16:
      return K % 64 == 0 ? kBF16w4 : K % 32 == 0 ? kBF16w2 : K % 16 == 0 ? kBF16w1 : kBadKind;
    case MOEB200_F32:
      return K % 32 == 0 ? kF32w2 : K % 16 == 0 ? kF32w1 : kBadKind;
  }
  return kBadKind;
}

// ---- shared / global vector loads ----------------------------------------------------------------
template <int NW>
__device__ __forceinline__ void lds(const uint8_t* p, uint32_t (&w)[NW]) {
  const uint32_t a = smem_u32(p);
  if constexpr (NW == 1) {
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(w[0]) : "r"(a));
  } else if constexpr (NW == 2) {
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(w[0]), "=r"(w[1]) : "r"(a));
  } else {
#pragma unroll
    for (int i = 0; i < NW; i += 4)
      asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                   : "=r"(w[i]), "=r"(w[i + 1]), "=r"(w[i + 2]), "=r"(w[i + 3])
                   : "r"(a + 4 * i));
  }
}

template <int NW>
__device__ __forceinline__ void ldg(const void* p, uint32_t (&w)[NW]) {
  if constexpr (NW == 1) {
    asm("ld.global.nc.u32 %0, [%1];" : "=r"(w[0]) : "l"(p));
  } else if constexpr (NW == 2) {
    asm("ld.global.nc.v2.u32 {%0,%1}, [%2];" : "=r"(w[0]), "=r"(w[1]) : "l"(p));
  } else {
#pragma unroll
    for (int i = 0; i < NW; i += 4)
      asm("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                   : "=r"(w[i]), "=r"(w[i + 1]), "=r"(w[i + 2]), "=r"(w[i + 3])
                   : "l"(static_cast<const uint8_t*>(p) + 16 * (i / 4)));
  }
}

// ---- B operand (activations of the lane's token(s)): NW words = 2*NW values, natural order ---------
template <typename AT, int NB>
struct BSrc {
  const AT* row[NB];  // null = token slot unused (zeros)

  template <int NW>
  __device__ __forceinline__ void load(int col, uint32_t (&xb)[NB][NW]) const {
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      if (row[nb] == nullptr) {
#pragma unroll
        for (int i = 0; i < NW; ++i) xb[nb][i] = 0u;
      } else {
        ldg<NW>(row[nb] + col, xb[nb]);
      }
    }
  }
};

// Scales of the lane's four rows (row tile rt, row g / g+8), read straight from the record (the 2-byte
// values of one row are contiguous, so consecutive chunks hit the same L1 sector).
struct Scales {
  const __half* p[2][2];
  __device__ __forceinline__ void load(int gi, float (&s)[2][2]) const {
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) s[rt][hh] = __half2float(__ldg(p[rt][hh] + gi));
  }
};

template <int NB>
__device__ __forceinline__ void fold_scaled(float (&tot)[2][NB][4], const float (&d)[2][NB][2][4],
                                            const float (&s)[2][2]) {
#pragma unroll
  for (int rt = 0; rt < 2; ++rt)
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      tot[rt][nb][0] = fmaf(s[rt][0], d[rt][nb][0][0] + d[rt][nb][1][0], tot[rt][nb][0]);
      tot[rt][nb][1] = fmaf(s[rt][0], d[rt][nb][0][1] + d[rt][nb][1][1], tot[rt][nb][1]);
      tot[rt][nb][2] = fmaf(s[rt][1], d[rt][nb][0][2] + d[rt][nb][1][2], tot[rt][nb][2]);
      tot[rt][nb][3] = fmaf(s[rt][1], d[rt][nb][0][3] + d[rt][nb][1][3], tot[rt][nb][3]);
    }
}

// ---- one 8*WPL-column (int4) / 4*WPL-column (int8, float) chunk per lane ----------------------------------
// st: stage (32 rows, stride rs; rows 0..15 = row tile 0, 16..31 = row tile 1); c: column of the chunk
// inside the stage; xb: the lane's activation words for the chunk; s: the rows' scales.

template <typename AT, int NB, int WPL>
__device__ __forceinline__ void chunk_int4(const uint8_t* st, int rs, int c, const uint32_t (&xb)[NB][4 * WPL],
                                           const float (&s)[2][2], float (&tot)[2][NB][4], int g, int t) {
  uint32_t wa[2][2][WPL];
#pragma unroll
  for (int rt = 0; rt < 2; ++rt)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) lds<WPL>(st + (rt * 16 + g + 8 * hh) * rs + c / 2 + 4 * WPL * t, wa[rt][hh]);
  float d[2][NB][2][4];
#pragma unroll
  for (int j = 0; j < WPL; ++j) {
    uint32_t p04[2][2], p15[2][2], p26[2][2], p37[2][2];
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) Dq<AT>::int4x8(wa[rt][hh][j], p04[rt][hh], p15[rt][hh], p26[rt][hh], p37[rt][hh]);
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      const uint32_t x0 = xb[nb][4 * j], x1 = xb[nb][4 * j + 1], x2 = xb[nb][4 * j + 2], x3 = xb[nb][4 * j + 3];
      const uint32_t b00 = prmt(x0, x2, 0x5410), b01 = prmt(x0, x2, 0x7632);  // (c, c+4), (c+1, c+5)
      const uint32_t b10 = prmt(x1, x3, 0x5410), b11 = prmt(x1, x3, 0x7632);  // (c+2, c+6), (c+3, c+7)
#pragma unroll
      for (int rt = 0; rt < 2; ++rt) {
        const uint32_t a0[4] = {p04[rt][0], p04[rt][1], p15[rt][0], p15[rt][1]};
        const uint32_t a1[4] = {p26[rt][0], p26[rt][1], p37[rt][0], p37[rt][1]};
        if (j == 0) {
          MmaOp<AT>::first(d[rt][nb][0], a0, b00, b01);
          MmaOp<AT>::first(d[rt][nb][1], a1, b10, b11);
        } else {
          MmaOp<AT>::run(d[rt][nb][0], a0, b00, b01);
          MmaOp<AT>::run(d[rt][nb][1], a1, b10, b11);
        }
      }
    }
  }
  fold_scaled<NB>(tot, d, s);
}

template <typename AT, int NB, int WPL>
__device__ __forceinline__ void chunk_int8(const uint8_t* st, int rs, int c, const uint32_t (&xb)[NB][2 * WPL],
                                           const float (&s)[2][2], float (&tot)[2][NB][4], int g, int t) {
  uint32_t wa[2][2][WPL];
#pragma unroll
  for (int rt = 0; rt < 2; ++rt)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) lds<WPL>(st + (rt * 16 + g + 8 * hh) * rs + c + 4 * WPL * t, wa[rt][hh]);
  float d[2][NB][2][4];
#pragma unroll
  for (int m = 0; m < WPL; ++m) {
    uint32_t p01[2][2], p23[2][2];
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) Dq<AT>::int8x4(wa[rt][hh][m], p01[rt][hh], p23[rt][hh]);
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int rt = 0; rt < 2; ++rt) {
        const uint32_t a[4] = {p01[rt][0], p01[rt][1], p23[rt][0], p23[rt][1]};
        if (m < 2)
          MmaOp<AT>::first(d[rt][nb][m & 1], a, xb[nb][2 * m], xb[nb][2 * m + 1]);
        else
          MmaOp<AT>::run(d[rt][nb][m & 1], a, xb[nb][2 * m], xb[nb][2 * m + 1]);
      }
  }
  if (WPL == 1) {  // only the first accumulator set was written
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int i = 0; i < 4; ++i) d[rt][nb][1][i] = 0.f;
  }
  fold_scaled<NB>(tot, d, s);
}

// Float records: WT is the stored element type; it is converted to the activation type when it
// differs (the reference materialises records in the activation dtype).
template <typename AT, typename WT, int NB, int WPL>
__device__ __forceinline__ void chunk_float(const uint8_t* st, int rs, int c, const uint32_t (&xb)[NB][2 * WPL],
                                            float (&tot)[2][NB][4], int g, int t) {
  constexpr int NWR = WPL * 4 * (int)sizeof(WT) / 4;  // weight words per row per lane per chunk
  uint32_t wr[2][2][NWR];
#pragma unroll
  for (int rt = 0; rt < 2; ++rt)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh)
      lds<NWR>(st + (rt * 16 + g + 8 * hh) * rs + (c + 4 * WPL * t) * (int)sizeof(WT), wr[rt][hh]);
#pragma unroll
  for (int m = 0; m < WPL; ++m) {
    uint32_t ap[2][2][2];  // [rt][hh][pair]
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        if constexpr (sizeof(WT) == 4) {
          const float* f = reinterpret_cast<const float*>(wr[rt][hh]) + 4 * m;
          ap[rt][hh][0] = Dq<AT>::pack_f32(f[0], f[1]);
          ap[rt][hh][1] = Dq<AT>::pack_f32(f[2], f[3]);
        } else if constexpr (std::is_same<WT, AT>::value) {
          ap[rt][hh][0] = wr[rt][hh][2 * m];
          ap[rt][hh][1] = wr[rt][hh][2 * m + 1];
        } else {
          const WT* v = reinterpret_cast<const WT*>(&wr[rt][hh][2 * m]);
          ap[rt][hh][0] = Dq<AT>::pack_f32(to_f32<WT>(v[0]), to_f32<WT>(v[1]));
          ap[rt][hh][1] = Dq<AT>::pack_f32(to_f32<WT>(v[2]), to_f32<WT>(v[3]));
        }
      }
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int rt = 0; rt < 2; ++rt) {
        const uint32_t a[4] = {ap[rt][0][0], ap[rt][1][0], ap[rt][0][1], ap[rt][1][1]};
        MmaOp<AT>::run(tot[rt][nb], a, xb[nb][2 * m], xb[nb][2 * m + 1]);
      }
  }
}

// ---- one pipeline step: the chunks of a stage, activations and scales loaded one chunk ahead ---------
// KIND selects the chunk routine; chunks alternate between two register sets so the next chunk's
// loads are in flight while the current chunk is multiplied.
template <typename AT, int NB, int KIND>
__device__ __forceinline__ void run_step(const uint8_t* st, int col0, int ncols, const BSrc<AT, NB>& B,
                                         const Scales& S, int gs, float (&tot)[2][NB][4], int g, int t) {
  constexpr bool I4 = KIND == kI4w2 || KIND == kI4w1;
  constexpr bool I8 = KIND == kI8w4 || KIND == kI8w2 || KIND == kI8w1;
  constexpr int WPL = (KIND == kI4w2 || KIND == kI8w2 || KIND == kF16w2 || KIND == kBF16w2 || KIND == kF32w2) ? 2
                      : (KIND == kI8w4 || KIND == kF16w4 || KIND == kBF16w4)                                   ? 4
                                                                                                                  : 1;
  constexpr int CH = I4 ? 32 * WPL : 16 * WPL;     // columns per chunk
  constexpr int NW = I4 ? 4 * WPL : 2 * WPL;       // activation words per lane per chunk
  constexpr int LOFF = I4 ? 8 * WPL : 4 * WPL;     // lane column offset inside a chunk
  constexpr int WT = KIND == kF32w2 || KIND == kF32w1 ? 2 : (KIND == kBF16w4 || KIND == kBF16w2 || KIND == kBF16w1) ? 1 : 0;
  constexpr int WTYPE = I4 ? MOEB200_I4 : I8 ? MOEB200_I8 : WT == 2 ? MOEB200_F32 : WT == 1 ? MOEB200_BF16 : MOEB200_F16;
  const int rs = gemv_row_stride(WTYPE);
  const int nch = ncols / CH;
  const int cpg = (I4 || I8) ? gs / CH : 1;
  const int g0 = (I4 || I8) ? col0 / gs : 0;
  auto chunk = [&](int ci, const uint32_t (&xv)[NB][NW], const float (&sv)[2][2]) {
    const int c = ci * CH;
    if constexpr (I4) {
      chunk_int4<AT, NB, WPL>(st, rs, c, xv, sv, tot, g, t);
    } else if constexpr (I8) {
      chunk_int8<AT, NB, WPL>(st, rs, c, xv, sv, tot, g, t);
    } else if constexpr (WT == 2) {
      chunk_float<AT, float, NB, WPL>(st, rs, c, xv, tot, g, t);
    } else if constexpr (WT == 1) {
      chunk_float<AT, __nv_bfloat16, NB, WPL>(st, rs, c, xv, tot, g, t);
    } else {
      chunk_float<AT, __half, NB, WPL>(st, rs, c, xv, tot, g, t);
    }
  };
  auto fetch = [&](int ci, uint32_t (&xv)[NB][NW], float (&sv)[2][2]) {
    B.template load<NW>(col0 + ci * CH + LOFF * t, xv);
    if constexpr (I4 || I8) S.load(g0 + (cpg == 1 ? ci : ci / cpg), sv);
  };
  uint32_t xa[NB][NW], xc[NB][NW];
  float sa[2][2] = {{0.f, 0.f}, {0.f, 0.f}}, sc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
  fetch(0, xa, sa);
  int ci = 0;
  for (; ci + 1 < nch; ci += 2) {
    fetch(ci + 1, xc, sc);
    chunk(ci, xa, sa);
    if (ci + 2 < nch) fetch(ci + 2, xa, sa);
    chunk(ci + 1, xc, sc);
  }
  if (ci < nch) chunk(ci, xa, sa);
}

// ---- tile description ---------------------------------------------------------------------------------
struct TileDesc {
  const uint8_t* rowbase[2];  // first row of each 16-row tile
  const uint8_t* sbase[2];    // first scale row of each 16-row tile (integer records)
  int32_t rstride;            // bytes per weight row
  int32_t sstride;            // bytes per scale row
  int32_t wtype, kind, gs, wbits;
  int32_t k_lo, k_hi;         // input columns of this K split
  int32_t step_cols, nsteps;
  int32_t item, r0;
};

// Input columns of one K split (a multiple of kSplitCols); splits past K are empty.
__device__ __forceinline__ int split_cols(int K, int ks_n) {
  return ks_n > 1 ? ((K / ks_n + kSplitCols - 1) / kSplitCols) * kSplitCols : K;
}

template <bool UP>
__device__ __forceinline__ void describe_tile(const GemvParams& p, int tile, int rb_per_item, int ks_n,
                                              TileDesc& d) {
  const int per_item = rb_per_item * ks_n;
  const int item = tile / per_item;
  const int rem = tile - item * per_item;
  const int ks = rem / rb_per_item;
  const int rb = rem - ks * rb_per_item;
  const Item it = p.items[item];
  const LayoutDev L = p.lay[it.slot];
  const int K = UP ? p.H : p.I;
  const bool isint = L.wtype == MOEB200_I4 || L.wtype == MOEB200_I8;
  d.item = item;
  d.wtype = L.wtype;
  d.wbits = wbits_of(L.wtype);
  d.gs = isint ? (UP ? L.gs_up : L.gs_dn) : 64;
  d.kind = kind_of(L.wtype, K, d.gs);
  d.rstride = K * d.wbits / 8;
  d.sstride = isint ? (K / d.gs) * 2 : 0;
  d.step_cols = kStepBytes * 8 / d.wbits;
  const int kc = split_cols(K, ks_n);
  d.k_lo = min(K, ks * kc);
  d.k_hi = min(K, d.k_lo + kc);
  d.nsteps = d.k_hi > d.k_lo ? (d.k_hi - d.k_lo + d.step_cols - 1) / d.step_cols : 0;
  const uint8_t* q = reinterpret_cast<const uint8_t*>(UP ? it.p_guq : it.p_dnq);
  const uint8_t* s = reinterpret_cast<const uint8_t*>(UP ? it.p_gus : it.p_dns);
  int rA, rB;
  if (UP) {
    d.r0 = rb * 16;
    rA = d.r0;
    rB = p.I + d.r0;
  } else {
    d.r0 = rb * 32;
    rA = d.r0;
    rB = d.r0 + 16;
  }
  d.rowbase[0] = q + (int64_t)rA * d.rstride;
  d.rowbase[1] = q + (int64_t)rB * d.rstride;
  d.sbase[0] = s + (int64_t)rA * d.sstride;
  d.sbase[1] = s + (int64_t)rB * d.sstride;
}

// Issue the bulk copies of one step (all 32 lanes take part; lane 0 arms the barrier first).
__device__ __forceinline__ void issue_step(const TileDesc& d, int step, uint8_t* stage, uint64_t* bar, int lane) {
  const int col0 = d.k_lo + step * d.step_cols;
  const int ncols = min(d.step_cols, d.k_hi - col0);
  const uint32_t seg = (uint32_t)(ncols * d.wbits / 8);
  if (lane == 0) mbar_arrive_expect_tx(bar, 32u * seg);
  __syncwarp();
  const int rt = lane >> 4, row = lane & 15;
  bulk_g2s(stage + lane * gemv_row_stride(d.wtype), d.rowbase[rt] + row * d.rstride + col0 * d.wbits / 8, seg, bar);
}

template <typename AT, int NB, bool UP, bool SPLIT>
__global__ void __launch_bounds__(kGemvMaxWarps * 32) gemv_kernel(const GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int nwarps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;

  if (UP && p.zero_acc) {  // the down phase reduces into acc; clear it first (grid-stride)
    const int64_t n = (int64_t)p.T * p.H;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
      p.acc[i] = 0.f;
  }

  const int sb = p.stage_bytes;
  uint8_t* stages = smem + warp * kGemvStages * sb;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + nwarps * kGemvStages * sb) + warp * kGemvStages;

  const int n_items = *p.n_items;
  const int rb_per_item = UP ? p.I / 16 : p.H / 32;
  const int ks_n = UP ? p.ksplit_up : p.ksplit_dn;
  const int n_tiles = n_items * rb_per_item * ks_n;
  const int gw = blockIdx.x * nwarps + warp;
  const int nw = gridDim.x * nwarps;
  if (gw >= n_tiles) return;

  // first tile of this warp with a non-empty K split (the producer and consumer walk the same list)
  int first = gw;
  TileDesc pd;
  describe_tile<UP>(p, first, rb_per_item, ks_n, pd);
  while (pd.nsteps == 0) {
    first += nw;
    if (first >= n_tiles) return;
    describe_tile<UP>(p, first, rb_per_item, ks_n, pd);
  }

  if (lane == 0) {
    for (int s = 0; s < kGemvStages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncwarp();

  int ptile = first, pstep = 0;
  auto produce = [&](int sidx) {
    if (ptile >= n_tiles) return;
    issue_step(pd, pstep, stages + sidx * sb, &bars[sidx], lane);
    if (++pstep == pd.nsteps) {
      pstep = 0;
      do {
        ptile += nw;
        if (ptile < n_tiles) describe_tile<UP>(p, ptile, rb_per_item, ks_n, pd);
      } while (ptile < n_tiles && pd.nsteps == 0);
    }
  };
  TileDesc cd = pd;  // the consumer starts on the same first tile
#pragma unroll
  for (int s = 0; s < kGemvStages; ++s) produce(s);

  int ctile = first, cstep = 0;
  float tot[2][NB][4];
  BSrc<AT, NB> B;
  Scales S;
  Item cit;
  auto begin_tile = [&]() {
    cit = p.items[cd.item];
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh)
        S.p[rt][hh] = reinterpret_cast<const __half*>(cd.sbase[rt] + (int64_t)(g + 8 * hh) * cd.sstride);
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      const int tk = g + 8 * nb;
      if (tk < cit.ntok) {
        const int j = cit.start + tk;
        if (UP) {
          const int tok = p.pos[j] / p.k;
          B.row[nb] = static_cast<const AT*>(p.x) + (int64_t)tok * p.H;
        } else {
          B.row[nb] = static_cast<const AT*>(p.h) + (int64_t)j * p.I;
        }
      } else {
        B.row[nb] = nullptr;
      }
#pragma unroll
      for (int rt = 0; rt < 2; ++rt)
#pragma unroll
        for (int i = 0; i < 4; ++i) tot[rt][nb][i] = 0.f;
    }
  };
  begin_tile();

  for (uint32_t it = 0;; ++it) {
    const int sidx = it % kGemvStages;
    if (!mbar_wait(&bars[sidx], (it / kGemvStages) & 1u, p.status)) return;
    const uint8_t* st = stages + sidx * sb;
    const int col0 = cd.k_lo + cstep * cd.step_cols;
    const int ncols = min(cd.step_cols, cd.k_hi - col0);
    switch (cd.kind) {
      case kI4w2: run_step<AT, NB, kI4w2>(st, col0, ncols, B, S, cd.gs, tot, g, t); break;
      case kI4w1: run_step<AT, NB, kI4w1>(st, col0, ncols, B, S, cd.gs, tot, g, t); break;
      case kI8w4: run_step<AT, NB, kI8w4>(st, col0, ncols, B, S, cd.gs, tot, g, t); break;
      case kI8w2: run_step<AT, NB, kI8w2>(st, col0, ncols, B, S, cd.gs, tot, g, t); break;
      case kI8w1: run_step<AT, NB, kI8w1>(st, col0, ncols, B, S, cd.gs, tot, g, t); break;
      case kF16w4: run_step<AT, NB, kF16w4>(st, col0, ncols, B, S, cd.gs, tot, g, t); break;
      case kF16w2: run_step<AT, NB, kF16w2>(st, col0, ncols, B, S, cd.gs, tot, g, t); break;
      case kF16w1: run_step<AT, NB, kF16w1>(st, col0, ncols, B, S, cd.gs, tot, g, t); break;
      case kBF16w4: run_step<AT, NB, kBF16w4>(st, col0, ncols, B, S, cd.gs, tot, g, t); break;
      case kBF16w2: run_step<AT, NB, kBF16w2>(st, col0, ncols, B, S, cd.gs, tot, g, t); break;
      case kBF16w1: run_step<AT, NB, kBF16w1>(st, col0, ncols, B, S, cd.gs, tot, g, t); break;
      case kF32w2: run_step<AT, NB, kF32w2>(st, col0, ncols, B, S, cd.gs, tot, g, t); break;
      case kF32w1: run_step<AT, NB, kF32w1>(st, col0, ncols, B, S, cd.gs, tot, g, t); break;
      default: break;
    }
    const bool last = (cstep + 1 == cd.nsteps);
    if (last) {
      // epilogue: c-fragment (row g | g+8, token 2t | 2t+1) per row tile and token block
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int tk = 8 * nb + 2 * t + (i & 1);
          if (tk >= cit.ntok) continue;
          const int rrow = g + 8 * (i >> 1);
          const int j = cit.start + tk;
          if (UP) {
            if constexpr (SPLIT) {
              float* prow = p.pre + (int64_t)j * 2 * p.I + cd.r0 + rrow;
              red_add_f32(prow, tot[0][nb][i]);
              red_add_f32(prow + p.I, tot[1][nb][i]);
            } else {
              const float hv = silu_mul(tot[0][nb][i], tot[1][nb][i]);
              static_cast<AT*>(p.h)[(int64_t)j * p.I + cd.r0 + rrow] = from_f32<AT>(hv);
            }
          } else {
            const int pos = p.pos[j];
            const int tok = pos / p.k;
            const float wv = p.wflat[pos];
            float* arow = p.acc + (int64_t)tok * p.H + cd.r0;
            red_add_f32(arow + rrow, wv * tot[0][nb][i]);
            red_add_f32(arow + 16 + rrow, wv * tot[1][nb][i]);
          }
        }
      if constexpr (UP && SPLIT) {
        // the last K split to arrive at this tile turns its 16 gate|up pre-activation rows into h
        __threadfence();
        __syncwarp();
        const int kc = split_cols(p.H, ks_n);
        const int ksplits = (p.H + kc - 1) / kc;  // non-empty splits
        int fin = 0;
        if (lane == 0) {
          int32_t* cnt = p.tile_cnt + (int64_t)cd.item * rb_per_item + cd.r0 / 16;
          fin = atomicAdd(cnt, 1) == ksplits - 1;
        }
        fin = __shfl_sync(0xffffffffu, fin, 0);
        if (fin) {
          __threadfence();
          for (int q = lane; q < 16 * cit.ntok; q += 32) {
            const int j = cit.start + q / 16, r = cd.r0 + (q & 15);
            const float* prow = p.pre + (int64_t)j * 2 * p.I;
            const float hv = silu_mul(__ldcg(prow + r), __ldcg(prow + p.I + r));
            static_cast<AT*>(p.h)[(int64_t)j * p.I + r] = from_f32<AT>(hv);
          }
        }
      }
    }
    __syncwarp();
    produce(sidx);  // refill the stage just consumed with the step kGemvStages ahead
    if (last) {
      cstep = 0;
      do {
        ctile += nw;
        if (ctile < n_tiles) describe_tile<UP>(p, ctile, rb_per_item, ks_n, cd);
      } while (ctile < n_tiles && cd.nsteps == 0);
      if (ctile >= n_tiles) break;
      begin_tile();
    } else {
      ++cstep;
    }
  }
}

template <typename AT>
__global__ void finalize_kernel(const float* __restrict__ acc, AT* __restrict__ out, int64_t n, int add) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = acc[i];
    out[i] = from_f32<AT>(add ? to_f32<AT>(out[i]) + v : v);
  }
}

// out[i] = sum over s = 0..G-1, in that order, of parts[s*n + i] (+ out[i] when add), cast once.
template <typename AT>
__global__ void combine_parts_kernel(const float* __restrict__ parts, int G, int64_t n, AT* __restrict__ out, int add) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float v = 0.f;
    for (int g = 0; g < G; ++g) v += parts[(int64_t)g * n + i];
    out[i] = from_f32<AT>(add ? to_f32<AT>(out[i]) + v : v);
  }
}

template <typename AT, int NB, bool UP, bool SPLIT>
cudaError_t launch_t(const GemvParams& p, int grid, int warps, cudaStream_t s) {
  const int smem = gemv_smem_bytes(p.stage_bytes, warps);
  auto kern = gemv_kernel<AT, NB, UP, SPLIT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, warps * 32, smem, s>>>(p);
  return cudaGetLastError();
}

template <typename AT, int NB, bool UP, bool SPLIT>
int occupancy_t(int smem, int warps) {
  auto kern = gemv_kernel<AT, NB, UP, SPLIT>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return 1;
  int nb = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, warps * 32, smem) != cudaSuccess) return 1;
  return nb;
}

// SPLIT: the up phase adds split-K partials into pre (the down phase always reads h).
template <typename AT, bool UP>
cudaError_t launch_phase(const GemvParams& p, int nb, int grid, int warps, cudaStream_t s) {
  if (UP && p.ksplit_up > 1)
    return nb == 2 ? launch_t<AT, 2, UP, true>(p, grid, warps, s) : launch_t<AT, 1, UP, true>(p, grid, warps, s);
  return nb == 2 ? launch_t<AT, 2, UP, false>(p, grid, warps, s) : launch_t<AT, 1, UP, false>(p, grid, warps, s);
}

template <typename AT>
int occupancy_at(int nb, bool up, bool split, int smem, int warps) {
  if (up) {
    if (split) return nb == 2 ? occupancy_t<AT, 2, true, true>(smem, warps) : occupancy_t<AT, 1, true, true>(smem, warps);
    return nb == 2 ? occupancy_t<AT, 2, true, false>(smem, warps) : occupancy_t<AT, 1, true, false>(smem, warps);
  }
  if (split) return nb == 2 ? occupancy_t<AT, 2, false, true>(smem, warps) : occupancy_t<AT, 1, false, true>(smem, warps);
  return nb == 2 ? occupancy_t<AT, 2, false, false>(smem, warps) : occupancy_t<AT, 1, false, false>(smem, warps);
}

}  // namespace

int gemv_occupancy(int act_type, int nb, bool up, bool split, int smem, int warps) {
  return act_type == MOEB200_BF16 ? occupancy_at<__nv_bfloat16>(nb, up, split, smem, warps)
                                  : occupancy_at<__half>(nb, up, split, smem, warps);
}

cudaError_t launch_gemv_up(const GemvParams& p, int act_type, int nb, int grid, int warps, cudaStream_t s) {
  return act_type == MOEB200_BF16 ? launch_phase<__nv_bfloat16, true>(p, nb, grid, warps, s)
                                  : launch_phase<__half, true>(p, nb, grid, warps, s);
}

cudaError_t launch_gemv_down(const GemvParams& p, int act_type, int nb, int grid, int warps, cudaStream_t s) {
  return act_type == MOEB200_BF16 ? launch_phase<__nv_bfloat16, false>(p, nb, grid, warps, s)
                                  : launch_phase<__half, false>(p, nb, grid, warps, s);
}

cudaError_t launch_combine_parts(const float* parts, int G, int64_t n, int act_type, void* out, int add,
                                 cudaStream_t s) {
  const int threads = 256;
  const int64_t nblk = (n + threads - 1) / threads;
  const int grid = (int)(nblk < 148 * 8 ? nblk : 148 * 8);
  if (act_type == MOEB200_BF16)
    combine_parts_kernel<__nv_bfloat16><<<grid, threads, 0, s>>>(parts, G, n, static_cast<__nv_bfloat16*>(out), add);
  else if (act_type == MOEB200_F16)
    combine_parts_kernel<__half><<<grid, threads, 0, s>>>(parts, G, n, static_cast<__half*>(out), add);
  else
    combine_parts_kernel<float><<<grid, threads, 0, s>>>(parts, G, n, static_cast<float*>(out), add);
  return cudaGetLastError();
}

cudaError_t launch_finalize(const float* acc, void* out, int act_type, int64_t n, int add, cudaStream_t s) {
  const int threads = 256;
  const int64_t nblk = (n + threads - 1) / threads;
  const int grid = (int)(nblk < 148 * 8 ? nblk : 148 * 8);
  if (act_type == MOEB200_BF16)
    finalize_kernel<__nv_bfloat16><<<grid, threads, 0, s>>>(acc, static_cast<__nv_bfloat16*>(out), n, add);
  else if (act_type == MOEB200_F16)
    finalize_kernel<__half><<<grid, threads, 0, s>>>(acc, static_cast<__half*>(out), n, add);
  else
    finalize_kernel<float><<<grid, threads, 0, s>>>(acc, static_cast<float*>(out), n, add);
  return cudaGetLastError();
}

}  // namespace moeb200
