// Grouped expert GEMV -- the decode path of the MoE layer on B200.
//
// Replaces the Triton grouped kernels of moelab (kernels.py `_grp4_up` 312-361, `_grp4_down`
// 363-396, `_grp8_up/_grp8_down` 667-740, `_grpf_up/_grpf_down` 398-451) with one warp-level
// pipeline per phase:
//
//   up   : h[j, r]  = silu(gate_r . x_tok(j)) * (up_r . x_tok(j))      for each pair j of an item
//   down : acc[t, r] += w_j * (down_r . h[j])                           (fp32 reduction = combine)
//
// Work is split into warp tiles (item, 32 weight rows): the up phase pairs 16 gate rows with the
// 16 matching up rows so SwiGLU happens in registers; the down phase takes 32 consecutive rows.
// Each warp streams its rows through its own ring of shared-memory stages filled by 1-D bulk TMA
// copies (one 128-byte row segment per lane per stage, padded row stride so the fragment reads
// are bank-conflict free), dequantises int4/int8 in registers straight into tensor-core A
// fragments, and multiplies them with the activations of up to 8*NB tokens of the item on
// mma.sync m16n8k16 with fp32 accumulators. The per-group fp16 scale is applied to the fp32
// partial of each chunk (a chunk never straddles a group), so the weights are never rounded.
// Rows are streamed once per item regardless of its token count.
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

__device__ __forceinline__ int stage_row_stride(int wtype) {
  return wtype == MOEB200_I4 ? 160 : wtype == MOEB200_I8 ? 192 : 144;
}

// Chunk kind for a matrix with K input columns and group size gs.
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
    asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(w[0]) : "l"(p));
  } else if constexpr (NW == 2) {
    asm volatile("ld.global.nc.v2.u32 {%0,%1}, [%2];" : "=r"(w[0]), "=r"(w[1]) : "l"(p));
  } else {
#pragma unroll
    for (int i = 0; i < NW; i += 4)
      asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                   : "=r"(w[i]), "=r"(w[i + 1]), "=r"(w[i + 2]), "=r"(w[i + 3])
                   : "l"(static_cast<const uint8_t*>(p) + 16 * (i / 4)));
  }
}

// B operand (activations) of the lane's token(s): NW 32-bit words starting at column `col`.
template <typename AT, int NB, int NW>
__device__ __forceinline__ void load_b(const AT* const (&xrow)[NB], int col, uint32_t (&xb)[NB][NW]) {
#pragma unroll
  for (int nb = 0; nb < NB; ++nb) {
    if (xrow[nb] != nullptr) {
      ldg<NW>(xrow[nb] + col, xb[nb]);
    } else {
#pragma unroll
      for (int i = 0; i < NW; ++i) xb[nb][i] = 0u;
    }
  }
}

// ---- one pipeline step of one warp tile, per weight kind ------------------------------------------
// st: stage buffer (32 rows, stride rs); rows 0..15 = row tile 0, 16..31 = row tile 1.
// col0: first input column of the step; ncols: columns in the step.
// sc: scale block of the tile in shared memory, [32 rows][ngroups] fp16.

template <typename AT, int NB, int WPL>
__device__ __forceinline__ void step_int4(const uint8_t* st, int rs, int col0, int ncols, const AT* const (&xrow)[NB],
                                          const __half* sc, int ngroups, int gs, float (&tot)[2][NB][4], int g,
                                          int t) {
  constexpr int CH = 32 * WPL;  // columns per chunk
  for (int c = 0; c < ncols; c += CH) {
    uint32_t wa[2][2][WPL];
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) lds<WPL>(st + (rt * 16 + g + 8 * hh) * rs + c / 2 + 4 * WPL * t, wa[rt][hh]);
    uint32_t xb[NB][4 * WPL];
    load_b<AT, NB, 4 * WPL>(xrow, col0 + c + 8 * WPL * t, xb);
    const int grp = (col0 + c) / gs;
    float s[2][2];
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) s[rt][hh] = __half2float(sc[(rt * 16 + g + 8 * hh) * ngroups + grp]);
    float d[2][NB][4];
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int i = 0; i < 4; ++i) d[rt][nb][i] = 0.f;
#pragma unroll
    for (int j = 0; j < WPL; ++j) {
      uint32_t p04[2][2], p15[2][2], p26[2][2], p37[2][2];
#pragma unroll
      for (int rt = 0; rt < 2; ++rt)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
          Dq<AT>::int4x8(wa[rt][hh][j], p04[rt][hh], p15[rt][hh], p26[rt][hh], p37[rt][hh]);
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        const uint32_t x0 = xb[nb][4 * j], x1 = xb[nb][4 * j + 1], x2 = xb[nb][4 * j + 2], x3 = xb[nb][4 * j + 3];
        const uint32_t b00 = prmt(x0, x2, 0x5410), b01 = prmt(x0, x2, 0x7632);  // (c, c+4), (c+1, c+5)
        const uint32_t b10 = prmt(x1, x3, 0x5410), b11 = prmt(x1, x3, 0x7632);  // (c+2, c+6), (c+3, c+7)
#pragma unroll
        for (int rt = 0; rt < 2; ++rt) {
          const uint32_t a0[4] = {p04[rt][0], p04[rt][1], p15[rt][0], p15[rt][1]};
          MmaOp<AT>::run(d[rt][nb], a0, b00, b01);
          const uint32_t a1[4] = {p26[rt][0], p26[rt][1], p37[rt][0], p37[rt][1]};
          MmaOp<AT>::run(d[rt][nb], a1, b10, b11);
        }
      }
    }
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        tot[rt][nb][0] = fmaf(s[rt][0], d[rt][nb][0], tot[rt][nb][0]);
        tot[rt][nb][1] = fmaf(s[rt][0], d[rt][nb][1], tot[rt][nb][1]);
        tot[rt][nb][2] = fmaf(s[rt][1], d[rt][nb][2], tot[rt][nb][2]);
        tot[rt][nb][3] = fmaf(s[rt][1], d[rt][nb][3], tot[rt][nb][3]);
      }
  }
}

template <typename AT, int NB, int WPL>
__device__ __forceinline__ void step_int8(const uint8_t* st, int rs, int col0, int ncols, const AT* const (&xrow)[NB],
                                          const __half* sc, int ngroups, int gs, float (&tot)[2][NB][4], int g,
                                          int t) {
  constexpr int CH = 16 * WPL;
  for (int c = 0; c < ncols; c += CH) {
    uint32_t wa[2][2][WPL];
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) lds<WPL>(st + (rt * 16 + g + 8 * hh) * rs + c + 4 * WPL * t, wa[rt][hh]);
    uint32_t xb[NB][2 * WPL];
    load_b<AT, NB, 2 * WPL>(xrow, col0 + c + 4 * WPL * t, xb);
    const int grp = (col0 + c) / gs;
    float s[2][2];
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) s[rt][hh] = __half2float(sc[(rt * 16 + g + 8 * hh) * ngroups + grp]);
    float d[2][NB][4];
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int i = 0; i < 4; ++i) d[rt][nb][i] = 0.f;
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
          MmaOp<AT>::run(d[rt][nb], a, xb[nb][2 * m], xb[nb][2 * m + 1]);
        }
    }
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        tot[rt][nb][0] = fmaf(s[rt][0], d[rt][nb][0], tot[rt][nb][0]);
        tot[rt][nb][1] = fmaf(s[rt][0], d[rt][nb][1], tot[rt][nb][1]);
        tot[rt][nb][2] = fmaf(s[rt][1], d[rt][nb][2], tot[rt][nb][2]);
        tot[rt][nb][3] = fmaf(s[rt][1], d[rt][nb][3], tot[rt][nb][3]);
      }
  }
}

// Float records: WT is the stored element type. When WT differs from the activation type the
// weights are converted to it (the reference materialises records in the activation dtype).
template <typename AT, typename WT, int NB, int WPL>
__device__ __forceinline__ void step_float(const uint8_t* st, int rs, int col0, int ncols,
                                           const AT* const (&xrow)[NB], float (&tot)[2][NB][4], int g, int t) {
  constexpr int CH = 16 * WPL;
  constexpr int NWR = WPL * 4 * (int)sizeof(WT) / 4;  // words of weights per row per lane per chunk
  for (int c = 0; c < ncols; c += CH) {
    uint32_t wr[2][2][NWR];
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh)
        lds<NWR>(st + (rt * 16 + g + 8 * hh) * rs + (c + 4 * WPL * t) * (int)sizeof(WT), wr[rt][hh]);
    uint32_t xb[NB][2 * WPL];
    load_b<AT, NB, 2 * WPL>(xrow, col0 + c + 4 * WPL * t, xb);
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
}

// ---- the pipelined warp-tile kernel -----------------------------------------------------------------
struct TileDesc {
  const uint8_t* rowbase[2];  // first row of each 16-row tile
  const uint8_t* sbase[2];    // first scale row of each tile (integer records)
  int64_t rstride;            // bytes per weight row
  int32_t sstride;            // bytes per scale row
  int32_t wtype, kind, gs, ngroups;
  int32_t step_cols, nsteps;
  int32_t item, r0;
};

template <bool UP>
__device__ __forceinline__ void describe_tile(const GemvParams& p, int64_t tile, int rb_per_item, TileDesc& d) {
  const int item = (int)(tile / rb_per_item);
  const int rb = (int)(tile % rb_per_item);
  const Item it = p.items[item];
  const LayoutDev L = p.lay[it.slot];
  const int K = UP ? p.H : p.I;
  const int wb = wbits_of(L.wtype);
  d.item = item;
  d.wtype = L.wtype;
  d.gs = UP ? L.gs_up : L.gs_dn;
  d.kind = kind_of(L.wtype, K, L.wtype == MOEB200_I4 || L.wtype == MOEB200_I8 ? d.gs : 64);
  d.rstride = (int64_t)K * wb / 8;
  d.ngroups = (L.wtype == MOEB200_I4 || L.wtype == MOEB200_I8) ? K / d.gs : 0;
  d.sstride = d.ngroups * 2;
  d.step_cols = kStepBytes * 8 / wb;
  d.nsteps = (K + d.step_cols - 1) / d.step_cols;
  const uint8_t* q = reinterpret_cast<const uint8_t*>(UP ? it.p_guq : it.p_dnq);
  const uint8_t* s = reinterpret_cast<const uint8_t*>(UP ? it.p_gus : it.p_dns);
  if (UP) {
    d.r0 = rb * 16;
    d.rowbase[0] = q + (int64_t)d.r0 * d.rstride;
    d.rowbase[1] = q + (int64_t)(p.I + d.r0) * d.rstride;
    d.sbase[0] = s + (int64_t)d.r0 * d.sstride;
    d.sbase[1] = s + (int64_t)(p.I + d.r0) * d.sstride;
  } else {
    d.r0 = rb * 32;
    d.rowbase[0] = q + (int64_t)d.r0 * d.rstride;
    d.rowbase[1] = q + (int64_t)(d.r0 + 16) * d.rstride;
    d.sbase[0] = s + (int64_t)d.r0 * d.sstride;
    d.sbase[1] = s + (int64_t)(d.r0 + 16) * d.sstride;
  }
}

// Issue the bulk copies of one step (all 32 lanes take part; lane 0 arms the barrier first).
__device__ __forceinline__ void issue_step(const TileDesc& d, int step, uint8_t* stage, uint8_t* sslot, uint64_t* bar,
                                           int lane) {
  const int K_cols = d.nsteps * d.step_cols;  // upper bound; the last step is clipped below
  (void)K_cols;
  const int wb = d.wtype == MOEB200_I4 ? 4 : d.wtype == MOEB200_I8 ? 8 : d.wtype == MOEB200_F32 ? 32 : 16;
  const int64_t Kfull = d.rstride * 8 / wb;
  const int col0 = step * d.step_cols;
  const int ncols = (int)(Kfull - col0 < d.step_cols ? Kfull - col0 : d.step_cols);
  const uint32_t seg = (uint32_t)(ncols * wb / 8);
  const bool scales = (step == 0) && d.ngroups > 0;
  const uint32_t sbytes = 16u * (uint32_t)d.sstride;
  if (lane == 0) mbar_arrive_expect_tx(bar, 32u * seg + (scales ? 2u * sbytes : 0u));
  __syncwarp();
  const int rt = lane >> 4, row = lane & 15;
  const int rs = stage_row_stride(d.wtype);
  bulk_g2s(stage + lane * rs, d.rowbase[rt] + row * d.rstride + (int64_t)col0 * wb / 8, seg, bar);
  if (scales && lane < 2) bulk_g2s(sslot + lane * sbytes, d.sbase[lane], sbytes, bar);
}

template <typename AT, int NB, bool UP>
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_kernel(const GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;

  if (UP && p.zero_acc) {  // the down phase reduces into acc; clear it first (grid-stride)
    const int64_t n = (int64_t)p.T * p.H;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
      p.acc[i] = 0.f;
  }

  const int wsm = gemv_warp_smem(p.scale_slot_bytes);
  uint8_t* wbase = smem + warp * wsm;
  uint8_t* stages = wbase;
  uint8_t* sslots = wbase + kGemvStages * kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kGemvWarps * wsm) + warp * kGemvStages;

  const int n_items = *p.n_items;
  const int rb_per_item = UP ? p.I / 16 : p.H / 32;
  const int64_t n_tiles = (int64_t)n_items * rb_per_item;
  const int64_t gw = (int64_t)blockIdx.x * kGemvWarps + warp;
  const int64_t nw = (int64_t)gridDim.x * kGemvWarps;
  if (gw >= n_tiles) return;

  if (lane == 0) {
    for (int s = 0; s < kGemvStages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncwarp();

  // producer cursor
  int64_t ptile = gw;
  int pstep = 0, pord = 0;
  TileDesc pd;
  describe_tile<UP>(p, ptile, rb_per_item, pd);
  auto produce = [&](int slot_stage) {
    if (ptile >= n_tiles) return;
    issue_step(pd, pstep, stages + slot_stage * kStageBytes, sslots + (pord % kGemvStages) * p.scale_slot_bytes,
               &bars[slot_stage], lane);
    if (++pstep == pd.nsteps) {
      pstep = 0;
      ++pord;
      ptile += nw;
      if (ptile < n_tiles) describe_tile<UP>(p, ptile, rb_per_item, pd);
    }
  };
#pragma unroll
  for (int s = 0; s < kGemvStages; ++s) produce(s);

  // consumer cursor
  int64_t ctile = gw;
  int cstep = 0, cord = 0;
  TileDesc cd;
  describe_tile<UP>(p, ctile, rb_per_item, cd);
  float tot[2][NB][4];
  const AT* xrow[NB];
  Item cit;
  auto begin_tile = [&]() {
    cit = p.items[cd.item];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      const int tk = g + 8 * nb;
      if (tk < cit.ntok) {
        const int j = cit.start + tk;
        if (UP) {
          const int tok = p.pos[j] / p.k;
          xrow[nb] = static_cast<const AT*>(p.x) + (int64_t)tok * p.H;
        } else {
          xrow[nb] = static_cast<const AT*>(p.h) + (int64_t)j * p.I;
        }
      } else {
        xrow[nb] = nullptr;
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
    const uint8_t* st = stages + sidx * kStageBytes;
    const __half* sc = reinterpret_cast<const __half*>(sslots + (cord % kGemvStages) * p.scale_slot_bytes);
    const int rs = stage_row_stride(cd.wtype);
    const int wb = cd.wtype == MOEB200_I4 ? 4 : cd.wtype == MOEB200_I8 ? 8 : cd.wtype == MOEB200_F32 ? 32 : 16;
    const int Kfull = (int)(cd.rstride * 8 / wb);
    const int col0 = cstep * cd.step_cols;
    const int ncols = min(cd.step_cols, Kfull - col0);
    switch (cd.kind) {
      case kI4w2: step_int4<AT, NB, 2>(st, rs, col0, ncols, xrow, sc, cd.ngroups, cd.gs, tot, g, t); break;
      case kI4w1: step_int4<AT, NB, 1>(st, rs, col0, ncols, xrow, sc, cd.ngroups, cd.gs, tot, g, t); break;
      case kI8w4: step_int8<AT, NB, 4>(st, rs, col0, ncols, xrow, sc, cd.ngroups, cd.gs, tot, g, t); break;
      case kI8w2: step_int8<AT, NB, 2>(st, rs, col0, ncols, xrow, sc, cd.ngroups, cd.gs, tot, g, t); break;
      case kI8w1: step_int8<AT, NB, 1>(st, rs, col0, ncols, xrow, sc, cd.ngroups, cd.gs, tot, g, t); break;
      case kF16w4: step_float<AT, __half, NB, 4>(st, rs, col0, ncols, xrow, tot, g, t); break;
      case kF16w2: step_float<AT, __half, NB, 2>(st, rs, col0, ncols, xrow, tot, g, t); break;
      case kF16w1: step_float<AT, __half, NB, 1>(st, rs, col0, ncols, xrow, tot, g, t); break;
      case kBF16w4: step_float<AT, __nv_bfloat16, NB, 4>(st, rs, col0, ncols, xrow, tot, g, t); break;
      case kBF16w2: step_float<AT, __nv_bfloat16, NB, 2>(st, rs, col0, ncols, xrow, tot, g, t); break;
      case kBF16w1: step_float<AT, __nv_bfloat16, NB, 1>(st, rs, col0, ncols, xrow, tot, g, t); break;
      case kF32w2: step_float<AT, float, NB, 2>(st, rs, col0, ncols, xrow, tot, g, t); break;
      case kF32w1: step_float<AT, float, NB, 1>(st, rs, col0, ncols, xrow, tot, g, t); break;
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
            const float hv = silu_mul(tot[0][nb][i], tot[1][nb][i]);
            static_cast<AT*>(p.h)[(int64_t)j * p.I + cd.r0 + rrow] = from_f32<AT>(hv);
          } else {
            const int pos = p.pos[j];
            const int tok = pos / p.k;
            const float wv = p.wflat[pos];
            float* arow = p.acc + (int64_t)tok * p.H + cd.r0;
            red_add_f32(arow + rrow, wv * tot[0][nb][i]);
            red_add_f32(arow + 16 + rrow, wv * tot[1][nb][i]);
          }
        }
    }
    __syncwarp();
    produce(sidx);  // refill the stage just consumed with the step kGemvStages ahead
    if (last) {
      cstep = 0;
      ++cord;
      ctile += nw;
      if (ctile >= n_tiles) break;
      describe_tile<UP>(p, ctile, rb_per_item, cd);
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

template <typename AT, int NB, bool UP>
cudaError_t launch_t(const GemvParams& p, int grid, cudaStream_t s) {
  const int smem = gemv_smem_bytes(p.scale_slot_bytes);
  auto kern = gemv_kernel<AT, NB, UP>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, kGemvWarps * 32, smem, s>>>(p);
  return cudaGetLastError();
}

}  // namespace

template <typename AT, int NB, bool UP>
int occupancy_t(int smem) {
  auto kern = gemv_kernel<AT, NB, UP>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return 1;
  int nb = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, kGemvWarps * 32, smem) != cudaSuccess) return 1;
  return nb;
}

int gemv_occupancy(int act_type, int nb, bool up, int smem) {
  if (act_type == MOEB200_BF16) {
    if (up) return nb == 2 ? occupancy_t<__nv_bfloat16, 2, true>(smem) : occupancy_t<__nv_bfloat16, 1, true>(smem);
    return nb == 2 ? occupancy_t<__nv_bfloat16, 2, false>(smem) : occupancy_t<__nv_bfloat16, 1, false>(smem);
  }
  if (up) return nb == 2 ? occupancy_t<__half, 2, true>(smem) : occupancy_t<__half, 1, true>(smem);
  return nb == 2 ? occupancy_t<__half, 2, false>(smem) : occupancy_t<__half, 1, false>(smem);
}

int gemv_smem_bytes(int scale_slot_bytes) {
  return kGemvWarps * gemv_warp_smem(scale_slot_bytes) + kGemvWarps * kGemvStages * 8;
}

cudaError_t launch_gemv_up(const GemvParams& p, int act_type, int nb, int grid, cudaStream_t s) {
  if (act_type == MOEB200_BF16)
    return nb == 2 ? launch_t<__nv_bfloat16, 2, true>(p, grid, s) : launch_t<__nv_bfloat16, 1, true>(p, grid, s);
  return nb == 2 ? launch_t<__half, 2, true>(p, grid, s) : launch_t<__half, 1, true>(p, grid, s);
}

cudaError_t launch_gemv_down(const GemvParams& p, int act_type, int nb, int grid, cudaStream_t s) {
  if (act_type == MOEB200_BF16)
    return nb == 2 ? launch_t<__nv_bfloat16, 2, false>(p, grid, s) : launch_t<__nv_bfloat16, 1, false>(p, grid, s);
  return nb == 2 ? launch_t<__half, 2, false>(p, grid, s) : launch_t<__half, 1, false>(p, grid, s);
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
