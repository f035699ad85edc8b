// Grouped expert GEMV -- the decode path of the MoE layer on B200.
//
// Replaces the Triton grouped kernels of moelab (kernels.py `_grp4_up` 312-361, `_grp4_down`
// 363-396, `_grp8_up/_grp8_down` 667-740, `_grpf_up/_grpf_down` 398-451):
//
//   up   : h[j, r]  = silu(gate_r . x_tok(j)) * (up_r . x_tok(j))      for each pair j of an item
//   down : acc[t, r] += w_j * (down_r . h[j])                           (fp32 reduction = combine)
//
// One persistent CTA per SM works through jobs = (work item, 256 weight rows, K split). Eight
// consumer warps own 32 rows each (up: 16 gate rows and the matching 16 up rows, so SwiGLU happens
// in registers). A producer warp streams the job's K range through kGemvStages shared-memory stages:
// per stage, tensor-map TMA loads (the map retargeted to the record on the device) bring a 128-byte
// swizzled tile of one kStepBytes segment of each of the 256 rows, and 1-D bulk copies the same
// columns of the item's token rows; the job's whole scale rows go to a double-buffered scale area
// with one or two bulk copies. Consumers dequantise in registers straight into mma.sync m16n8k16
// A fragments and multiply them with up to 8*NB tokens:
//   int4/int8 records: (q - 8) (int8: q) is exact in fp16 and bf16; the tensor cores sum its exact
//     products with the activations of one scale group in fp32, and the group's fp32 partial is
//     multiplied by its fp16 scale (exact in fp32) -- one rounding fewer than materialising
//     w = (q - 8) * s in the activation dtype first, and no per-weight scale multiply;
//   float records: converted to the activation type when the types differ.
// Small batches split K over jobs: the up phase then adds fp32 partial pre-activations into
// pre[j, 0:2I] (gate | up) and the job whose split of a row block arrives last (a per-(item, row
// block) counter) forms h = silu(gate) * up for its rows, so the down phase always reads h.
#include <algorithm>
#include <type_traits>

#include "gemv.cuh"
#include "tma.cuh"

namespace moeb200 {

namespace {

// Tensor-map templates of a launch: for each precision slot, the weight field of the phase
// (gate_up.q or down.q) as a 2-D uint8 tensor [rows][row bytes] read in 128-byte x R-row boxes with
// 128-byte swizzle; the kernel swaps in each record's address (tensormap.replace) per job.
struct alignas(64) TmaTemplates {
  CUtensorMap m[4];
};

enum Kind : int32_t {
  kI4w2 = 0, kI4w1, kI8w4, kI8w2, kI8w1, kF16w4, kF16w2, kF16w1, kBF16w4, kBF16w2, kBF16w1, kF32w2, kF32w1,
  kBadKind
};

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

// ---- shared-memory helpers ---------------------------------------------------------------------------
template <int NW>
__device__ __forceinline__ void lds(uint32_t a, uint32_t (&w)[NW]) {
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

// Weight words of one row from the swizzled weight tile: bytes [o, o + 4*NW) of the row's
// kStepBytes step, given the swizzled offsets of the 16-byte pieces that hold them (so0: first piece, so1:
// second piece when the access spans 32 bytes).
template <int NW>
__device__ __forceinline__ void ldw(uint32_t row, uint32_t so0, uint32_t so1, uint32_t (&w)[NW]) {
  if constexpr (NW <= 4) {
    lds<NW>(row + so0, w);
  } else {
    static_assert(NW == 8, "weight accesses span one or two 16-byte pieces");
    uint32_t a[4], b[4];
    lds<4>(row + so0, a);
    lds<4>(row + so1, b);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      w[i] = a[i];
      w[4 + i] = b[i];
    }
  }
}

// Offset of byte o (o < kStepBytes) of a row's step inside the weight tile: each 128 bytes of the
// step are a separate TMA box column, 32 KB apart; inside a box, 16-byte piece c of row R sits at
// piece c ^ (R % 8) (128-byte swizzle). Every row a lane touches has R % 8 == g.
__device__ __forceinline__ uint32_t swz(uint32_t o, uint32_t g) {
  return ((o >> 7) << 15) | ((((o >> 4) & 7u) ^ g) << 4) | (o & 15u);
}

__device__ __forceinline__ uint32_t lds_u16(uint32_t a) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
  return v;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Named barrier of the consumer warps only (the producer warp never takes part).
__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kGemvCons * 32) : "memory");
}

// ---- scales of the lane's four rows (row tile rt, row g / g+8) for one group -------------------------
struct Scales {
  uint32_t row[2][2];  // shared address of each row's first scale in the job's scale area
  __device__ __forceinline__ void f32(int gi, float (&s)[2][2]) const {
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh)
        s[rt][hh] = __half2float(__ushort_as_half((unsigned short)lds_u16(row[rt][hh] + 2 * gi)));
  }
};

template <int NB, int NA>
__device__ __forceinline__ void fold_one(float (&tot)[2][NB][4], const float (&d)[2][NA][4], const float (&s)[2][2]) {
#pragma unroll
  for (int rt = 0; rt < 2; ++rt)
#pragma unroll
    for (int nb = 0; nb < NA; ++nb) {
      tot[rt][nb][0] = fmaf(s[rt][0], d[rt][nb][0], tot[rt][nb][0]);
      tot[rt][nb][1] = fmaf(s[rt][0], d[rt][nb][1], tot[rt][nb][1]);
      tot[rt][nb][2] = fmaf(s[rt][1], d[rt][nb][2], tot[rt][nb][2]);
      tot[rt][nb][3] = fmaf(s[rt][1], d[rt][nb][3], tot[rt][nb][3]);
    }
}
// ---- one chunk per lane --------------------------------------------------------------------------------
// wr[rt][hh]: shared address of the start of the lane's weight row g + 8*hh of row tile rt in the
// weight tile; so0/so1: swizzled offsets of the lane's bytes of the chunk in those rows (ldw);
// xb[nb]: the lane's activation words of the chunk (token g + 8*nb). Only the first NA <= NB token
// blocks are computed: a job whose item has at most 8 tokens skips the empty second block.

// int4: chunk = 32*WPL columns, lane t holds columns [c + 8*WPL*t, +8*WPL) as WPL words per row.
// The exact (q - 8) products of a group are summed in fp32 and the group's partial is scaled once.
template <typename AT, int NB, int NA, int WPL>
__device__ __forceinline__ void chunk_int4(const uint32_t (&wr)[2][2], uint32_t so0, uint32_t so1,
                                           const uint32_t (&xb)[NA][4 * WPL], const Scales& S, int gi,
                                           float (&tot)[2][NB][4]) {
  uint32_t wa[2][2][WPL];
#pragma unroll
  for (int rt = 0; rt < 2; ++rt)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) ldw<WPL>(wr[rt][hh], so0, so1, wa[rt][hh]);
  {
    float d[2][NA][4];
#pragma unroll
    for (int j = 0; j < WPL; ++j) {
      uint32_t p04[2][2], p15[2][2], p26[2][2], p37[2][2];
#pragma unroll
      for (int rt = 0; rt < 2; ++rt)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
          Dq<AT>::int4x8(wa[rt][hh][j], p04[rt][hh], p15[rt][hh], p26[rt][hh], p37[rt][hh]);
#pragma unroll
      for (int nb = 0; nb < NA; ++nb) {
        const uint32_t x0 = xb[nb][4 * j], x1 = xb[nb][4 * j + 1], x2 = xb[nb][4 * j + 2], x3 = xb[nb][4 * j + 3];
        const uint32_t b00 = prmt(x0, x2, 0x5410), b01 = prmt(x0, x2, 0x7632);
        const uint32_t b10 = prmt(x1, x3, 0x5410), b11 = prmt(x1, x3, 0x7632);
#pragma unroll
        for (int rt = 0; rt < 2; ++rt) {
          const uint32_t a0[4] = {p04[rt][0], p04[rt][1], p15[rt][0], p15[rt][1]};
          const uint32_t a1[4] = {p26[rt][0], p26[rt][1], p37[rt][0], p37[rt][1]};
          if (j == 0)
            MmaOp<AT>::first(d[rt][nb], a0, b00, b01);
          else
            MmaOp<AT>::run(d[rt][nb], a0, b00, b01);
          MmaOp<AT>::run(d[rt][nb], a1, b10, b11);
        }
      }
    }
    float s[2][2];
    S.f32(gi, s);
    fold_one<NB, NA>(tot, d, s);
  }
}

// int8: chunk = 16*WPL columns, lane t holds columns [c + 4*WPL*t, +4*WPL) as WPL words per row.
template <typename AT, int NB, int NA, int WPL>
__device__ __forceinline__ void chunk_int8(const uint32_t (&wr)[2][2], uint32_t so0, uint32_t so1,
                                           const uint32_t (&xb)[NA][2 * WPL], const Scales& S, int gi,
                                           float (&tot)[2][NB][4]) {
  uint32_t wa[2][2][WPL];
#pragma unroll
  for (int rt = 0; rt < 2; ++rt)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) ldw<WPL>(wr[rt][hh], so0, so1, wa[rt][hh]);
  {
    float d[2][NA][4];
#pragma unroll
    for (int m = 0; m < WPL; ++m) {
      uint32_t p01[2][2], p23[2][2];
#pragma unroll
      for (int rt = 0; rt < 2; ++rt)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) Dq<AT>::int8x4(wa[rt][hh][m], p01[rt][hh], p23[rt][hh]);
#pragma unroll
      for (int nb = 0; nb < NA; ++nb)
#pragma unroll
        for (int rt = 0; rt < 2; ++rt) {
          const uint32_t a[4] = {p01[rt][0], p01[rt][1], p23[rt][0], p23[rt][1]};
          if (m == 0)
            MmaOp<AT>::first(d[rt][nb], a, xb[nb][2 * m], xb[nb][2 * m + 1]);
          else
            MmaOp<AT>::run(d[rt][nb], a, xb[nb][2 * m], xb[nb][2 * m + 1]);
        }
    }
    float s[2][2];
    S.f32(gi, s);
    fold_one<NB, NA>(tot, d, s);
  }
}

// Float records: WT is the stored element type; it is converted to the activation type when it
// differs (the reference materialises records in the activation dtype). Chunk = 16*WPL columns,
// lane t holds columns [c + 4*WPL*t, +4*WPL).
template <typename AT, typename WT, int NB, int NA, int WPL>
__device__ __forceinline__ void chunk_float(const uint32_t (&wr)[2][2], uint32_t so0, uint32_t so1,
                                            const uint32_t (&xb)[NA][2 * WPL], float (&tot)[2][NB][4]) {
  constexpr int NWR = WPL * 4 * (int)sizeof(WT) / 4;  // weight words per row per lane per chunk
  uint32_t wv[2][2][NWR];
#pragma unroll
  for (int rt = 0; rt < 2; ++rt)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) ldw<NWR>(wr[rt][hh], so0, so1, wv[rt][hh]);
#pragma unroll
  for (int m = 0; m < WPL; ++m) {
    uint32_t ap[2][2][2];  // [rt][hh][pair]
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        if constexpr (sizeof(WT) == 4) {
          const float* f = reinterpret_cast<const float*>(wv[rt][hh]) + 4 * m;
          ap[rt][hh][0] = Dq<AT>::pack_f32(f[0], f[1]);
          ap[rt][hh][1] = Dq<AT>::pack_f32(f[2], f[3]);
        } else if constexpr (std::is_same<WT, AT>::value) {
          ap[rt][hh][0] = wv[rt][hh][2 * m];
          ap[rt][hh][1] = wv[rt][hh][2 * m + 1];
        } else {
          const WT* v = reinterpret_cast<const WT*>(&wv[rt][hh][2 * m]);
          ap[rt][hh][0] = Dq<AT>::pack_f32(to_f32<WT>(v[0]), to_f32<WT>(v[1]));
          ap[rt][hh][1] = Dq<AT>::pack_f32(to_f32<WT>(v[2]), to_f32<WT>(v[3]));
        }
      }
#pragma unroll
    for (int nb = 0; nb < NA; ++nb)
#pragma unroll
      for (int rt = 0; rt < 2; ++rt) {
        const uint32_t a[4] = {ap[rt][0][0], ap[rt][1][0], ap[rt][0][1], ap[rt][1][1]};
        MmaOp<AT>::run(tot[rt][nb], a, xb[nb][2 * m], xb[nb][2 * m + 1]);
      }
  }
}

// ---- one stage: its chunks, the lane's activation words read from the stage's token rows ----------
// rowoff[rt][hh]: offset of the lane's row in the weight tile (row index * 128).
template <typename AT, int NB, int NA, int KIND>
__device__ __forceinline__ void run_stage(uint32_t wtile, const uint32_t (&rowoff)[2][2], uint32_t bbase,
                                          int bstride, int ntok, int ncols, int col0, int gs, int g0,
                                          const Scales& S, float (&tot)[2][NB][4], int g, int t) {
  constexpr bool I4 = KIND == kI4w2 || KIND == kI4w1;
  constexpr bool I8 = KIND == kI8w4 || KIND == kI8w2 || KIND == kI8w1;
  constexpr int WPL = (KIND == kI4w2 || KIND == kI8w2 || KIND == kF16w2 || KIND == kBF16w2 || KIND == kF32w2) ? 2
                      : (KIND == kI8w4 || KIND == kF16w4 || KIND == kBF16w4)                                   ? 4
                                                                                                                  : 1;
  constexpr int CH = I4 ? 32 * WPL : 16 * WPL;  // columns per chunk
  constexpr int NW = I4 ? 4 * WPL : 2 * WPL;    // activation words per lane per chunk
  constexpr int LOFF = I4 ? 8 * WPL : 4 * WPL;  // lane column offset inside a chunk
  constexpr int WT = KIND == kF32w2 || KIND == kF32w1 ? 2 : (KIND == kBF16w4 || KIND == kBF16w2 || KIND == kBF16w1) ? 1 : 0;
  constexpr int W2 = I4 ? 1 : I8 ? 2 : WT == 2 ? 8 : 4;  // weight bytes per column, times 2
  const int nch = ncols / CH;
  uint32_t wr[2][2];
#pragma unroll
  for (int rt = 0; rt < 2; ++rt)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) wr[rt][hh] = wtile + rowoff[rt][hh];
  uint32_t brow[NA];
  bool bon[NA];
#pragma unroll
  for (int nb = 0; nb < NA; ++nb) {
    bon[nb] = g + 8 * nb < ntok;
    brow[nb] = bbase + (g + 8 * nb) * bstride + LOFF * t * 2;
  }
  const uint32_t lo = LOFF * t * W2 / 2;  // the lane's first byte inside a chunk
  // group of each chunk, advanced without divisions (a chunk never straddles a group)
  const int cpg = (I4 || I8) ? gs / CH : 1;
  int gi = (I4 || I8) ? col0 / gs - g0 : 0, cc = (I4 || I8) ? (col0 % gs) / CH : 0;
#pragma unroll 2
  for (int ci = 0; ci < nch; ++ci) {
    uint32_t xb[NA][NW];
#pragma unroll
    for (int nb = 0; nb < NA; ++nb) {
      if (bon[nb]) {
        lds<NW>(brow[nb] + ci * CH * 2, xb[nb]);
      } else {
#pragma unroll
        for (int i = 0; i < NW; ++i) xb[nb][i] = 0u;
      }
    }
    const uint32_t o = ci * (CH * W2 / 2) + lo;
    const uint32_t so0 = swz(o, g), so1 = swz(o + 16, g);
    if constexpr (I4) {
      chunk_int4<AT, NB, NA, WPL>(wr, so0, so1, xb, S, gi, tot);
    } else if constexpr (I8) {
      chunk_int8<AT, NB, NA, WPL>(wr, so0, so1, xb, S, gi, tot);
    } else if constexpr (WT == 2) {
      chunk_float<AT, float, NB, NA, WPL>(wr, so0, so1, xb, tot);
    } else if constexpr (WT == 1) {
      chunk_float<AT, __nv_bfloat16, NB, NA, WPL>(wr, so0, so1, xb, tot);
    } else {
      chunk_float<AT, __half, NB, NA, WPL>(wr, so0, so1, xb, tot);
    }
    if (++cc == cpg) {
      cc = 0;
      ++gi;
    }
  }
}

// ---- jobs ----------------------------------------------------------------------------------------------
// Input columns of one K split (a multiple of kSplitCols); splits past K are empty.
__host__ __device__ __forceinline__ int split_cols(int K, int ks_n) {
  return ks_n > 1 ? ((K / ks_n + kSplitCols - 1) / kSplitCols) * kSplitCols : K;
}

struct Job {
  const uint8_t* q;  // weight field of the record (gate_up or down)
  const uint8_t* s;  // scale field (integer records)
  int32_t item, rb, ks, start, ntok, slot;
  int32_t kind, gs, wbits;
  int32_t r0, nrow;          // up: first gate row and gate rows (up rows mirror them); down: rows
  int32_t k_lo, k_hi;        // input columns of this K split
  int32_t step_cols, nsteps;
  int32_t rstride, sstride;  // bytes per weight row / scale row in the record
  int32_t g0, ngr, sst;      // first group held (0), groups per scale row, scale-area row stride
};

__device__ __forceinline__ int job_item(int job, int rb_per_item, int ks_n) { return job / (rb_per_item * ks_n); }

// A job as the producer announces it to the consumers, in the shared-memory slot of the job's first
// stage (job < 0: no more jobs).
struct alignas(16) JobSlot {
  Item it;
  int32_t job;
  int32_t _pad[3];
};
static_assert(sizeof(JobSlot) == 64, "JobSlot layout");

// Item of a job (a global load: callers fetch it one job ahead).
__device__ __forceinline__ Item load_item(const GemvParams& p, int job, int n_jobs, int rb_per_item, int ks_n) {
  Item it{};
  if (job < n_jobs) it = p.items[job_item(job, rb_per_item, ks_n)];
  return it;
}

template <bool UP>
__device__ __forceinline__ void describe_job(const GemvParams& p, int job, const Item& it, int rb_per_item, int ks_n,
                                             Job& d) {
  const int per_item = rb_per_item * ks_n;
  const int item = job / per_item;
  const int rem = job - item * per_item;
  const int ks = rem / rb_per_item;
  const int rb = rem - ks * rb_per_item;
  const LayoutDev L = p.lay[it.slot];
  const int K = UP ? p.H : p.I;
  const bool isint = L.wtype == MOEB200_I4 || L.wtype == MOEB200_I8;
  d.item = item;
  d.rb = rb;
  d.ks = ks;
  d.slot = it.slot;
  d.start = it.start;
  d.ntok = it.ntok;
  d.wbits = gemv_wbits(L.wtype);
  d.gs = isint ? (UP ? L.gs_up : L.gs_dn) : 64;
  d.kind = kind_of(L.wtype, K, d.gs);
  d.rstride = K * d.wbits / 8;
  d.sstride = isint ? (K / d.gs) * 2 : 0;
  d.step_cols = kStepBytes * 8 / d.wbits;
  const int kc = split_cols(K, ks_n);
  d.k_lo = min(K, ks * kc);
  d.k_hi = min(K, d.k_lo + kc);
  d.nsteps = d.k_hi > d.k_lo ? (d.k_hi - d.k_lo + d.step_cols - 1) / d.step_cols : 0;
  d.q = reinterpret_cast<const uint8_t*>(UP ? it.p_guq : it.p_dnq);
  d.s = reinterpret_cast<const uint8_t*>(UP ? it.p_gus : it.p_dns);
  if (UP) {
    d.r0 = rb * (kGemvJobRows / 2);
    d.nrow = min(kGemvJobRows / 2, p.I - d.r0);
  } else {
    d.r0 = rb * kGemvJobRows;
    d.nrow = min(kGemvJobRows, p.H - d.r0);
  }
  d.g0 = 0;  // scale areas hold whole scale rows: groups are indexed absolutely
  d.ngr = isint ? K / d.gs : 0;
  d.sst = d.sstride;
}

// ---- the kernel -----------------------------------------------------------------------------------------
template <typename AT, int NB, bool UP, bool SPLIT>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(const GemvParams p, const __grid_constant__ TmaTemplates tm) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte aligned base: the 128-byte swizzle of the weight tiles repeats every 1024 bytes
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;

  uint8_t* stages = smem;
  uint8_t* sarea = smem + kGemvStages * p.stage_bytes;
  uint8_t* sdesc = sarea + 2 * p.s_bytes;  // 128-byte tensor-map staging of the producer
  uint64_t* bars = reinterpret_cast<uint64_t*>(sdesc + 128);
  uint64_t* full = bars;                      // [stages] stage landed
  uint64_t* empty = bars + kGemvStages;       // [stages] stage consumed by every consumer warp
  uint64_t* sfull = bars + 2 * kGemvStages;   // [2] scale area landed
  uint64_t* sempty = sfull + 2;               // [2] scale area released
  int32_t* bcast = reinterpret_cast<int32_t*>(sempty + 2);
  JobSlot* jslot = reinterpret_cast<JobSlot*>(sempty + 4);  // [stages], 16-byte aligned

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGemvStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kGemvCons);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sfull[s], 1);
      mbar_init(&sempty[s], kGemvCons);
    }
    fence_mbar_init();
  }
  __syncthreads();
  // everything above touched shared memory only; the previous kernel's outputs are read below
  chain_wait();
  chain_release();

  if (UP && p.zero_acc) {  // the down phase reduces into acc; clear it first (grid-stride)
    const int64_t n = (int64_t)p.T * p.H;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
      p.acc[i] = 0.f;
  }

  const int n_items = *p.n_items;
  const int rb_per_item = UP ? (p.I + kGemvJobRows / 2 - 1) / (kGemvJobRows / 2)
                             : (p.H + kGemvJobRows - 1) / kGemvJobRows;
  const int ks_n = UP ? p.ksplit_up : p.ksplit_dn;
  const int n_jobs = n_items * rb_per_item * ks_n;

  if (warp == kGemvCons) {
    // ---------------- producer warp ----------------
    uint32_t it = 0, sj = 0, jn = 0;
    bool ok = true;
    // Job order: a CTA's first two jobs are blockIdx.x and blockIdx.x + gridDim.x (no draw on the
    // path of small launches); every further job is drawn from the launch's job counter (jobs are
    // numbered largest records first), so CTAs that draw short jobs take more of them and the CTAs
    // finish together. The next job is drawn, and its item loaded, while the current one streams.
    int32_t* ctr = p.job_next + (UP ? 0 : 1);
    int jpre = blockIdx.x;  // next job index to describe
    int taken = 0;          // jobs described so far
    Item ipre = load_item(p, jpre, n_jobs, rb_per_item, ks_n);
    auto draw = [&]() -> int {
      if (++taken == 1) return (int)(blockIdx.x + gridDim.x);
      int j = 0;
      if (lane == 0) j = (int)(2 * gridDim.x) + atomicAdd(ctr, 1);
      return __shfl_sync(0xffffffffu, j, 0);
    };
    // describes the next non-empty job (its index in j, its item in jit)
    auto next_job = [&](int& j, Item& jit, Job& out) -> bool {
      while (jpre < n_jobs) {
        j = jpre;
        jit = ipre;
        describe_job<UP>(p, j, jit, rb_per_item, ks_n, out);
        jpre = draw();
        ipre = load_item(p, jpre, n_jobs, rb_per_item, ks_n);
        if (out.nsteps > 0) return true;
      }
      return false;
    };
    // tensor maps of the jobs' weight fields: a ring of kMapRing per CTA. Each job's map is pointed
    // at its record while the previous job streams (after that job's first stage is issued), so
    // small jobs do not wait for the retarget; a slot is rewritten kMapRing jobs after its last use,
    // when every copy through it has landed (issuing a stage waits for the stage kGemvStages back,
    // and every job issues at least one stage)
    constexpr uint32_t kMapRing = 2 * kGemvStages;
    static_assert(kMapRing <= kTmapSlots && kMapRing > kGemvStages, "tensor-map ring");
    auto map_slot = [&](uint32_t n) {
      return reinterpret_cast<uint64_t>(p.tmap_ws) + (uint64_t)(blockIdx.x * kTmapSlots + (n % kMapRing)) * 128;
    };
    int job = 0;
    Item jit{};
    Job d;
    bool has = next_job(job, jit, d);
    uint64_t gdesc = 0;
    if (has) {
      gdesc = map_slot(jn++);
      retarget_tmap(tm.m[d.slot], smem_u32(sdesc), gdesc, d.q, lane);
    }
    while (has && ok) {
      int jnext = 0;
      Item jitn{};
      Job dn;
      bool hn = false;
      uint64_t gnext = 0;
      // token rows of the item (one per lane)
      const AT* brow = nullptr;
      if (lane < d.ntok) {
        const int j = d.start + lane;
        brow = UP ? static_cast<const AT*>(p.x) + (int64_t)(p.pos[j] / p.k) * p.H
                  : static_cast<const AT*>(p.h) + (int64_t)j * p.I;
      }
      if (d.ngr > 0) {
        // the job's scale area: whole scale rows of its gate (or down) rows at row 0 and of its up
        // rows at row 128 -- contiguous blocks of the record, one bulk copy each
        const int par = sj & 1;
        if (sj >= 2) ok = mbar_wait(&sempty[par], ((sj >> 1) - 1) & 1, p.status);
        if (!ok) break;
        if (lane == 0) {
          uint8_t* sa = sarea + par * p.s_bytes;
          const uint32_t blk = (uint32_t)(d.nrow * d.sstride);
          mbar_arrive_expect_tx(&sfull[par], UP ? 2 * blk : blk);
          bulk_g2s(sa, d.s + (int64_t)d.r0 * d.sstride, blk, &sfull[par]);
          if (UP)
            bulk_g2s(sa + (kGemvJobRows / 2) * d.sstride, d.s + (int64_t)(p.I + d.r0) * d.sstride, blk, &sfull[par]);
        }
        ++sj;
      }
      for (int step = 0; step < d.nsteps; ++step, ++it) {
        const int sidx = it % kGemvStages;
        if (it >= kGemvStages) ok = mbar_wait(&empty[sidx], ((it / kGemvStages) - 1) & 1, p.status);
        if (!ok) break;
        const int col0 = d.k_lo + step * d.step_cols;
        const int ncols = min(d.step_cols, d.k_hi - col0);
        const uint32_t bseg = (uint32_t)(ncols * (int)sizeof(AT));
        const uint32_t wst = smem_u32(stages + sidx * p.stage_bytes);
        if (lane == 0) {
          if (step == 0) {  // announce the job with its first stage (published by the arrive below)
            jslot[sidx].it = jit;
            jslot[sidx].job = job;
          }
          // the weight tile: whole boxes land (rows or bytes past the tensor read as zeros)
          mbar_arrive_expect_tx(&full[sidx], kGemvWBytes + d.ntok * bseg);
          const int xb = col0 * d.wbits / 8;  // first byte of the step in each row (a multiple of 128)
#pragma unroll
          for (int bc = 0; bc < kStepBytes / 128; ++bc) {
            const uint32_t wc = wst + bc * kGemvBoxCol;
            if (UP) {
              tma2d(wc, gdesc, xb + 128 * bc, d.r0, &full[sidx]);                // gate rows -> R 0..127
              tma2d(wc + 128 * 128, gdesc, xb + 128 * bc, p.I + d.r0, &full[sidx]);  // up rows -> R 128..255
            } else {
              tma2d(wc, gdesc, xb + 128 * bc, d.r0, &full[sidx]);                // rows -> R 0..255
            }
          }
        }
        __syncwarp();
        if (lane < d.ntok)
          bulk_g2s(stages + sidx * p.stage_bytes + kGemvWBytes + lane * p.b_stride, brow + col0, bseg, &full[sidx]);
        if (step == 0) {  // the next job's map, while this job's first stage lands
          hn = next_job(jnext, jitn, dn);
          if (hn) {
            gnext = map_slot(jn++);
            retarget_tmap(tm.m[dn.slot], smem_u32(sdesc), gnext, dn.q, lane);
          }
        }
      }
      d = dn;
      jit = jitn;
      job = jnext;
      gdesc = gnext;
      has = hn;
    }
    // the CTA must not exit with copies in flight: wait for the last stages issued (consumed
    // already in the normal flow; after a failed wait they may still be landing)
    for (uint32_t q = it > kGemvStages ? it - kGemvStages : 0; q < it; ++q)
      mbar_wait(&full[q % kGemvStages], (q / kGemvStages) & 1, nullptr);
    // then tell the consumers that no job follows: job -1 in the slot of the next stage, once that
    // stage's previous use has been consumed (after a failed wait the consumers time out instead)
    if (ok) {
      const int sidx = it % kGemvStages;
      if (it >= kGemvStages) ok = mbar_wait(&empty[sidx], ((it / kGemvStages) - 1) & 1, p.status);
      if (ok && lane == 0) {
        jslot[sidx].job = -1;
        mbar_arrive(&full[sidx]);
      }
    }
    return;
  }

  // ---------------- consumer warps ----------------
  uint32_t it = 0, sj = 0;
  bool failed = false;  // a bounded wait gave up (status word set): stop after the current job
  const uint32_t st0 = smem_u32(stages);
  const uint32_t sa0 = smem_u32(sarea);
  // rows of this lane in the weight tile (R * 128): up = gate rows 16w.. and up rows 128 + 16w..;
  // down = rows 32w..32w+31
  uint32_t rowoff[2][2];
#pragma unroll
  for (int rt = 0; rt < 2; ++rt)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int R = UP ? rt * 128 + 16 * warp + g + 8 * hh : 32 * warp + 16 * rt + g + 8 * hh;
      rowoff[rt][hh] = R * 128;
    }
  while (!failed) {
    // the next job is announced in the slot of its first stage: wait for that stage, read the job
    {
      const int sidx = it % kGemvStages;
      if (!mbar_wait(&full[sidx], (it / kGemvStages) & 1, p.status)) break;
    }
    const JobSlot& js = jslot[it % kGemvStages];
    const int job = js.job;
    if (job < 0) break;  // no more jobs
    Job d;
    describe_job<UP>(p, job, js.it, rb_per_item, ks_n, d);
    // the down epilogue's token and weight of each of the lane's fragment tokens, loaded now
    int etok[NB][2];
    float ew[NB][2];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        etok[nb][e] = -1;
        ew[nb][e] = 0.f;
        const int tk = 8 * nb + 2 * t + e;
        if (!UP && tk < d.ntok) {
          const int pos = p.pos[d.start + tk];
          etok[nb][e] = pos / p.k;
          ew[nb][e] = p.wflat[pos];
        }
      }
    const bool mine = UP ? 16 * warp < d.nrow : 32 * warp < d.nrow;  // this warp has rows in the job
    Scales S{};
    int par = 0;
    if (d.ngr > 0) {
      par = sj & 1;
      if (!mbar_wait(&sfull[par], (sj >> 1) & 1, p.status)) failed = true;
      const uint32_t sa = sa0 + par * p.s_bytes;
#pragma unroll
      for (int rt = 0; rt < 2; ++rt)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          // scale-area row of the lane's row: up = gate rows at 0.., up rows at 128..; down = rows
          const int m = UP ? rt * (kGemvJobRows / 2) + 16 * warp + g + 8 * hh : 32 * warp + 16 * rt + g + 8 * hh;
          S.row[rt][hh] = sa + m * d.sst;
        }
    }
    float tot[2][NB][4];
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int i = 0; i < 4; ++i) tot[rt][nb][i] = 0.f;
    for (int step = 0; step < d.nsteps && !failed; ++step, ++it) {
      const int sidx = it % kGemvStages;
      if (step > 0 && !mbar_wait(&full[sidx], (it / kGemvStages) & 1, p.status)) {
        failed = true;  // finish this job's barriers with the other consumer warps, then stop
        break;
      }
      const int col0 = d.k_lo + step * d.step_cols;
      const int ncols = min(d.step_cols, d.k_hi - col0);
      const uint32_t wtile = st0 + sidx * p.stage_bytes;
      const uint32_t bbase = wtile + kGemvWBytes;
      if (mine) {
        // token blocks holding tokens of this job (NB = 2 kernels skip the second for items of <= 8)
        const bool one = NB == 2 && d.ntok <= 8;
        switch (d.kind) {
#define MOEB200_STAGE(K)                                                                                        \
  case K:                                                                                                       \
    if (one)                                                                                                    \
      run_stage<AT, NB, 1, K>(wtile, rowoff, bbase, p.b_stride, d.ntok, ncols, col0, d.gs, d.g0, S, tot, g, t); \
    else                                                                                                        \
      run_stage<AT, NB, NB, K>(wtile, rowoff, bbase, p.b_stride, d.ntok, ncols, col0, d.gs, d.g0, S, tot, g, t); \
    break;
          MOEB200_STAGE(kI4w2)
          MOEB200_STAGE(kI4w1)
          MOEB200_STAGE(kI8w4)
          MOEB200_STAGE(kI8w2)
          MOEB200_STAGE(kI8w1)
          MOEB200_STAGE(kF16w4)
          MOEB200_STAGE(kF16w2)
          MOEB200_STAGE(kF16w1)
          MOEB200_STAGE(kBF16w4)
          MOEB200_STAGE(kBF16w2)
          MOEB200_STAGE(kBF16w1)
          MOEB200_STAGE(kF32w2)
          MOEB200_STAGE(kF32w1)
#undef MOEB200_STAGE
          default:
            break;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[sidx]);
    }
    if (d.ngr > 0) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&sempty[par]);
      ++sj;
    }
    // epilogue: c-fragment (row g | g+8, token 2t | 2t+1) per row tile and token block
    if (mine) {
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int tk = 8 * nb + 2 * t + (i & 1);
          if (tk >= d.ntok) continue;
          const int rrow = g + 8 * (i >> 1);
          const int j = d.start + tk;
          if (UP) {
            if (16 * warp + rrow >= d.nrow) continue;
            const int r = d.r0 + 16 * warp + rrow;  // gate row; its up row is I + r
            if constexpr (SPLIT) {
              float* prow = p.pre + ((int64_t)d.ks * p.pre_rows + j) * 2 * p.I + r;  // this split's slice
              prow[0] = tot[0][nb][i];
              prow[p.I] = tot[1][nb][i];
            } else {
              const float hv = silu_mul(tot[0][nb][i], tot[1][nb][i]);
              static_cast<AT*>(p.h)[(int64_t)j * p.I + r] = from_f32<AT>(hv);
            }
          } else {
            float* arow = p.acc + (int64_t)etok[nb][i & 1] * p.H + d.r0 + 32 * warp;
            const float wv = ew[nb][i & 1];
            red_add_f32(arow + rrow, wv * tot[0][nb][i]);
            red_add_f32(arow + 16 + rrow, wv * tot[1][nb][i]);
          }
        }
    }
    if constexpr (UP && SPLIT) {
      // the last K split of this row block to arrive turns the block's pre-activations into h
      __threadfence();
      consumers_sync();
      const int kc = split_cols(p.H, ks_n);
      const int ksplits = (p.H + kc - 1) / kc;  // non-empty splits
      if (threadIdx.x == 0) {
        int32_t* cnt = p.tile_cnt + (int64_t)d.item * rb_per_item + d.rb;
        *bcast = atomicAdd(cnt, 1) == ksplits - 1;
      }
      consumers_sync();
      const int fin = *bcast;
      consumers_sync();  // bcast is reused by the next job
      if (fin) {
        __threadfence();
        for (int q = threadIdx.x; q < d.nrow * d.ntok; q += kGemvCons * 32) {
          const int j = d.start + q / d.nrow, r = d.r0 + q % d.nrow;
          // the splits' partial sums, added in split order (the same sum on every run)
          float gv = 0.f, uv = 0.f;
          for (int sp = 0; sp < ksplits; ++sp) {
            const float* prow = p.pre + ((int64_t)sp * p.pre_rows + j) * 2 * p.I;
            gv += __ldcg(prow + r);
            uv += __ldcg(prow + p.I + r);
          }
          const float hv = silu_mul(gv, uv);
          static_cast<AT*>(p.h)[(int64_t)j * p.I + r] = from_f32<AT>(hv);
        }
      }
    }
  }
}

template <typename AT>
__global__ void finalize_kernel(const float* __restrict__ acc, AT* __restrict__ out, int64_t n, int add) {
  chain_wait();
  chain_release();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = acc[i];
    out[i] = from_f32<AT>(add ? to_f32<AT>(out[i]) + v : v);
  }
}

// out[i] = sum over s = 0..G-1, in that order, of parts[s*n + i] (+ out[i] when add), cast once.
template <typename AT>
__global__ void combine_parts_kernel(const float* __restrict__ parts, int G, int64_t n, AT* __restrict__ out, int add) {
  chain_wait();
  chain_release();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float v = 0.f;
    for (int g = 0; g < G; ++g) v += parts[(int64_t)g * n + i];
    out[i] = from_f32<AT>(add ? to_f32<AT>(out[i]) + v : v);
  }
}

template <typename AT, int NB, bool UP, bool SPLIT>
cudaError_t launch_t(const GemvParams& p, const TmaTemplates& tm, int grid, int smem, cudaStream_t s) {
  auto kern = gemv_kernel<AT, NB, UP, SPLIT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  return launch_chained(kern, dim3(grid), dim3(kGemvThreads), (size_t)smem, s, p, tm);
}

template <typename AT, bool UP>
cudaError_t launch_phase(const GemvParams& p, const TmaTemplates& tm, int nb, int grid, int smem, cudaStream_t s) {
  if (UP && p.ksplit_up > 1)
    return nb == 2 ? launch_t<AT, 2, UP, true>(p, tm, grid, smem, s) : launch_t<AT, 1, UP, true>(p, tm, grid, smem, s);
  return nb == 2 ? launch_t<AT, 2, UP, false>(p, tm, grid, smem, s) : launch_t<AT, 1, UP, false>(p, tm, grid, smem, s);
}

bool is_int_type(int wt) { return wt == MOEB200_I4 || wt == MOEB200_I8; }

// A K split must cover whole groups and whole chunks: kSplitCols is a multiple of every group size.
bool split_ok(const moeb200_layout* L, int nlay, int K, bool up, int ks) {
  if (K < ks * kSplitCols / 2) return false;
  for (int i = 0; i < nlay; ++i)
    if (is_int_type(L[i].wtype) && kSplitCols % (up ? L[i].gs_up : L[i].gs_dn)) return false;
  return true;
}

// Shared-memory geometry of a phase (kGemvStages stages, 2 scale areas, tensor-map staging, barriers, 1024
// bytes of alignment slack); returns its bytes.
int phase_smem(GemvParams& p, const moeb200_layout* lays, int nlay, int nb, int K, bool up, int ks) {
  int bst = 0, sst = 0;
  for (int i = 0; i < nlay; ++i) {
    bst = std::max(bst, gemv_b_stride(lays[i].wtype));
    if (is_int_type(lays[i].wtype)) {  // a job's scale area holds whole scale rows
      const int gs = up ? lays[i].gs_up : lays[i].gs_dn;
      sst = std::max(sst, K / gs * 2);
    }
  }
  (void)ks;
  p.b_stride = bst;
  p.b_rows = 8 * nb;
  p.stage_bytes = (kGemvWBytes + p.b_rows * bst + 1023) / 1024 * 1024;
  p.s_bytes = (kGemvJobRows * sst + 127) / 128 * 128;
  // barriers: full/empty per stage, sfull/sempty (2 each), the broadcast word (16 bytes), a 64-byte
  // job slot per stage
  return kGemvStages * p.stage_bytes + 2 * p.s_bytes + 128 + (2 * kGemvStages + 6) * 8 + kGemvStages * 64 + 1024;
}

cudaError_t plan_and_launch(GemvParams& p, const moeb200_layout* lays, int nlay, int act, int nb, int max_items,
                            int n_pairs, int max_split_pairs, bool up, cudaStream_t s) {
  const int sms = num_sms_cached();
  const int K = up ? p.H : p.I;
  const int rows = up ? p.I : p.H;
  const int rpj = up ? kGemvJobRows / 2 : kGemvJobRows;
  const int64_t jobs1 = (int64_t)max_items * ((rows + rpj - 1) / rpj);
  // split K while the jobs would not give every SM four of them (jobs of different records differ
  // several-fold in bytes; more, smaller jobs balance the CTAs; up: only with room for pre)
  int ks = 1;
  const bool can_split = !up || (max_items <= max_split_pairs && n_pairs <= max_split_pairs && p.pre != nullptr);
  // up: one pre slice per split (the pointer-table entry points size their slices with capi.cu
  // table_split_slices, which mirrors this loop without split_ok)
  const int ks_cap = up && p.pre_slices > 0 ? p.pre_slices : kMaxKSplit;
  while (can_split && ks < ks_cap && jobs1 * ks < (int64_t)sms && split_ok(lays, nlay, K, up, ks * 2)) ks *= 2;
  if (up)
    p.ksplit_up = ks;
  else
    p.ksplit_dn = ks;
  const int smem = phase_smem(p, lays, nlay, nb, K, up, ks);
  if (smem > 227 * 1024) return cudaErrorInvalidConfiguration;
  TmaTemplates tm{};
  for (int i = 0; i < nlay; ++i) {
    const int row_bytes = K * gemv_wbits(lays[i].wtype) / 8;
    cudaError_t e = tma_weight_template(&tm.m[i], row_bytes, up ? 2 * p.I : p.H, up ? kGemvJobRows / 2 : kGemvJobRows,
                                    p.tmap_ws);
    if (e != cudaSuccess) return e;
  }
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(std::min(sms, kGemvMaxGrid), jobs1 * ks));
  if (act == MOEB200_BF16)
    return up ? launch_phase<__nv_bfloat16, true>(p, tm, nb, grid, smem, s)
              : launch_phase<__nv_bfloat16, false>(p, tm, nb, grid, smem, s);
  return up ? launch_phase<__half, true>(p, tm, nb, grid, smem, s) : launch_phase<__half, false>(p, tm, nb, grid, smem, s);
}

}  // namespace

cudaError_t launch_gemv_phases(GemvParams& p, const moeb200_layout* lays, int nlay, int act_type, int nb,
                               int max_items, int n_pairs, int max_split_pairs, cudaStream_t s) {
  p.ksplit_up = p.ksplit_dn = 1;
  cudaError_t e = trace_mark(0, s);
  if (e != cudaSuccess) return e;
  e = plan_and_launch(p, lays, nlay, act_type, nb, max_items, n_pairs, max_split_pairs, true, s);
  if (e != cudaSuccess) return e;
  e = trace_mark(1, s);
  if (e != cudaSuccess) return e;
  e = plan_and_launch(p, lays, nlay, act_type, nb, max_items, n_pairs, max_split_pairs, false, s);
  if (e != cudaSuccess) return e;
  return trace_mark(2, s);
}

cudaError_t launch_combine_parts(const float* parts, int G, int64_t n, int act_type, void* out, int add,
                                 cudaStream_t s) {
  const int threads = 256;
  const int64_t nblk = (n + threads - 1) / threads;
  const dim3 grid((unsigned)(nblk < 148 * 8 ? nblk : 148 * 8));
  if (act_type == MOEB200_BF16)
    return launch_chained(combine_parts_kernel<__nv_bfloat16>, grid, dim3(threads), 0, s, parts, G, n,
                          static_cast<__nv_bfloat16*>(out), add);
  if (act_type == MOEB200_F16)
    return launch_chained(combine_parts_kernel<__half>, grid, dim3(threads), 0, s, parts, G, n,
                          static_cast<__half*>(out), add);
  return launch_chained(combine_parts_kernel<float>, grid, dim3(threads), 0, s, parts, G, n,
                        static_cast<float*>(out), add);
}

cudaError_t launch_finalize(const float* acc, void* out, int act_type, int64_t n, int add, cudaStream_t s) {
  const int threads = 256;
  const int64_t nblk = (n + threads - 1) / threads;
  const dim3 grid((unsigned)(nblk < 148 * 8 ? nblk : 148 * 8));
  if (act_type == MOEB200_BF16)
    return launch_chained(finalize_kernel<__nv_bfloat16>, grid, dim3(threads), 0, s, acc,
                          static_cast<__nv_bfloat16*>(out), n, add);
  if (act_type == MOEB200_F16)
    return launch_chained(finalize_kernel<__half>, grid, dim3(threads), 0, s, acc, static_cast<__half*>(out), n, add);
  return launch_chained(finalize_kernel<float>, grid, dim3(threads), 0, s, acc, static_cast<float*>(out), n, add);
}

}  // namespace moeb200
