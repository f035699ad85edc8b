/*
 * moeb200 -- C ABI of the B200-native MoE-layer hot path.
 *
 * A drop-in for the compute behind moelab's `OffloadedExperts` module (moelab/runtime.py:1094-1112)
 * and for the transformers router it keeps (`parent.gate`, moelab/loader.py:222-223). Every entry
 * point takes plain device pointers, sizes and a cudaStream_t passed as void*; none allocates, and
 * apart from moeb200_check_workspace none synchronises or reads device memory on the host, so those
 * calls can be recorded in a CUDA graph.
 * Every entry point returns a status (0 = OK); moeb200_last_error() gives the message of the last
 * failure on the calling thread.
 *
 * Data formats follow moelab exactly:
 *  - expert records: one uint8 blob per (layer, expert, precision) with the field table of
 *    moelab/store.py:76-115 (gate_up [2I,H] then down [H,I]; int8/int4 add fp16 scales per group
 *    of gs input columns; int4 packs two values per byte, low nibble = even column, stored +8).
 *  - routing: top_k_index int64 [T,k], top_k_weights float32 [T,k] (transformers TopKRouter).
 *  - precision levels: uint8 [T,k], 0 = most precise precision of the store (moelab/policy.py).
 */
#ifndef MOEB200_H
#define MOEB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------------------------- */
enum {
  MOEB200_OK = 0,
  MOEB200_ERR_INVALID = 1,     /* bad argument: shape, type, alignment or null pointer        */
  MOEB200_ERR_UNSUPPORTED = 2, /* valid for moelab, not handled by these kernels (message says) */
  MOEB200_ERR_CUDA = 3,        /* a CUDA runtime call or kernel launch failed                 */
  MOEB200_ERR_WORKSPACE = 4    /* workspace smaller than the *_workspace() query returned      */
};

/* ---- element types ------------------------------------------------------------------------ */
enum { MOEB200_F32 = 0, MOEB200_F16 = 1, MOEB200_BF16 = 2, MOEB200_I8 = 3, MOEB200_I4 = 4 };

/* Field table of one expert record (mirror of moelab/store.py:76-115 `record_layout`).
 * wtype: F32/F16/BF16 for float records, I8/I4 for quantised ones.
 * Float records: off_gu_q = offset of gate_up, off_dn_q = offset of down, *_s = -1, gs_* = 0. */
typedef struct {
  int32_t wtype;
  int32_t hidden;
  int32_t inter;
  int32_t gs_up;
  int32_t gs_dn;
  int32_t _pad;
  int64_t off_gu_q;
  int64_t off_gu_s;
  int64_t off_dn_q;
  int64_t off_dn_s;
  int64_t record_bytes;
} moeb200_layout;

/* Precision policy (mirror of moelab/policy.py:20-58 PrecisionPolicy, plus the build's threshold
 * rule). mode: 0 "hi" (every pair level 0), 1 "lo" (every pair level 2), 2 "hobbit",
 * 3 "threshold" (level 0 if the pair's router weight >= thr, else level 2).
 * t_mid / t2 < 0 mean "unset" (None in the reference). */
typedef struct {
  int32_t mode;
  float t1;
  float t_mid;
  float t2;
  float thr;
} moeb200_policy;

/* Device table of resident expert records for one layer (mirror of moelab/fullgraph.py:43-98
 * DeviceTable): table[p * E + e] = device address of expert e's record at precision slot p
 * (0 = not resident). Precision slots are ordered most precise first, as moelab's store lists.
 * tma_base (no reference counterpart): a device address at or below every record the table can
 * hold, with every record address a multiple of 4096 above it; the fused decode kernel reads
 * records through tensor maps based there (0 = not given: that kernel is not used). */
typedef struct {
  int32_t n_prec;
  int32_t num_experts;
  moeb200_layout layout[4];
  const int64_t* table;
  int64_t tma_base;
} moeb200_expert_table;

const char* moeb200_version(void);

/* Copies the last error message of the calling thread into buf (always NUL-terminated).
 * Returns the status of that failure. */
int moeb200_last_error(char* buf, size_t n);

/* Number of SMs of the current device (cached per device). */
int moeb200_num_sms(void);

/* Expert-product path of the following moeb200_experts_forward calls on the calling thread
 * (no reference counterpart): 0 = automatic (tcgen05 GEMM when T*k >= 40*E; else the warp-streamed
 * GEMV of path 4 for T <= 8 where it applies, else the two-launch grouped GEMV), 1 = grouped GEMV, 2 = tcgen05 GEMM (needs H and I multiples of 128), 3 = the fused
 * one-launch decode kernel (int4/int8 records with group size 64 or float records of the activation
 * type, H and I multiples of 64 up to 2048, a table with tma_base; refused with
 * MOEB200_ERR_UNSUPPORTED where it does not apply), 4 = the warp-streamed grouped GEMV (items of at
 * most 8 pairs; int4/int8 records with group size 64 or float records of the activation type;
 * H and I multiples of 512; x 16-byte aligned; refused with MOEB200_ERR_UNSUPPORTED otherwise). */
int moeb200_set_path(int32_t path);
/* Pairs per grouped-GEMV work item for the following moeb200_experts_forward calls on the calling
 * thread (no reference counterpart): 0 = automatic (16 when T >= 64, else 8), 8 or 16. A larger
 * item streams an expert's record once for more tokens at the cost of more multiplies per byte.
 * The fused decode kernel always works on items of 8; 16 makes the automatic path skip it. */
int moeb200_set_item_tokens(int32_t nt);

/* Measurement hooks (no reference counterpart). Between trace_begin and trace_end, every
 * grouped-expert call of the calling thread records CUDA events (owned by the library) on its
 * stream before the gate/up phase, between the two phases and after the down phase.
 * trace_end synchronises on them and returns the summed phase times (ms) and the call count;
 * it is for benchmarks, not for captured graphs. */
int moeb200_trace_begin(void);
int moeb200_trace_end(float* up_ms, float* down_ms, int32_t* calls);
/* Measurement hook (no reference counterpart): the expert-product path the calling thread's last
 * moeb200_experts_forward(_part) call took -- 1 grouped GEMV, 2 tcgen05 GEMM, 3 fused decode kernel
 * (its whole launch is traced as the gate/up phase), 4 warp-streamed grouped GEMV -- or 0 before
 * the first call. */
int moeb200_path_used(void);

/* ---- router --------------------------------------------------------------------------------
 * Replaces transformers OlmoeTopKRouter / Qwen3MoeTopKRouter / Qwen3NextTopKRouter.forward
 * (olmoe/modeling_olmoe.py:350-359, qwen3_moe/modeling_qwen3_moe.py:254-272,
 *  qwen3_next/modeling_qwen3_next.py:761-779): logits = h . Wr^T accumulated in fp32 and rounded
 * to the model dtype, + bias[e] (fp32, optional synthetic skew), probs = softmax in fp32 over all
 * E, top-k with ties broken by the lower expert index, optional renormalisation of the k weights.
 * h [T,H] and wr [E,H] are act_type (F16/BF16/F32). probs [T,E] may be NULL. logits [T,E] (may be
 * NULL) receives the model-dtype-rounded logits before the bias, as float32.
 * If policy != NULL the HOBBIT / threshold levels of each pair are also written to level [T,k]
 * and skip [T,k] (uint8, 1 = skipped). */
int moeb200_router(const void* h, const void* wr, const float* bias, int32_t act_type, int32_t T, int32_t H,
                   int32_t E, int32_t k, int32_t renorm, float* probs, float* w, int64_t* idx, float* logits,
                   const moeb200_policy* policy, uint8_t* level, uint8_t* skip, void* ws, size_t ws_bytes,
                   void* stream);
size_t moeb200_router_workspace(int32_t T, int32_t E);
/* Router with a Qwen3-Next shared expert folded in as one more routed pair per token (no reference
 * counterpart: transformers runs the shared expert beside the routed ones,
 * qwen3_next/modeling_qwen3_next.py:789-801, and moelab leaves it there). wr holds E + 1 rows:
 * the E router rows, then the shared expert's gate row (shared_expert_gate.weight). w, idx and
 * level / skip are [T, k + 1]: the k routed pairs as moeb200_router gives them, then the pair
 * (expert E, sigmoid(x . wg) with the logit rounded to the activation dtype, level shared_level,
 * not skipped). probs stays [T, E]; logits, when given, is [T, E + 1]; size the workspace with
 * moeb200_router_workspace(T, E + 1). An expert table with E + 1 experts whose expert E holds the
 * shared MLP's record (at the precision slot shared_level selects) then computes the routed and
 * shared experts in the same launches. */
int moeb200_router_shared(const void* h, const void* wr, const float* bias, int32_t act_type, int32_t T, int32_t H,
                          int32_t E, int32_t k, int32_t renorm, int32_t shared_level, float* probs, float* w,
                          int64_t* idx, float* logits, const moeb200_policy* policy, uint8_t* level, uint8_t* skip,
                          void* ws, size_t ws_bytes, void* stream);

/* ---- precision levels ----------------------------------------------------------------------
 * Replaces PrecisionPolicy.levels / levels_one (moelab/policy.py:110-137) and the device version
 * gpu_levels (moelab/fullgraph.py:101-114): w [T,k] fp32 -> level [T,k] uint8 in {0,1,2},
 * skip [T,k] uint8 (may be NULL). */
int moeb200_levels(const float* w, int32_t T, int32_t k, const moeb200_policy* policy, uint8_t* level,
                   uint8_t* skip, void* stream);

/* Per-expert precision vote of the reference's multi-token path (PrecisionPolicy.expert_level,
 * moelab/policy.py:148-154, applied per expert by MoERuntime._decide_general,
 * moelab/runtime.py:476-488): over the kept pairs of each expert, the expert's level is the most
 * precise L in {0, 1} asked for by at least hi_vote of them, else 2; level [T,k] is rewritten in
 * place so that every kept pair carries its expert's level. skip may be NULL. E <= 16384. */
int moeb200_levels_vote(const int64_t* idx, uint8_t* level, const uint8_t* skip, int32_t T, int32_t k, int32_t E,
                        double hi_vote, void* stream);

/* ---- dispatch --------------------------------------------------------------------------------
 * Replaces the routing part of MoERuntime._decide_general (moelab/runtime.py:459-492): pairs
 * (t, j) not skipped are flattened to p = t*k + j and sorted stably
 *   - by expert:                counts_e [E], pos_e [T*k]   (= flat_pos[order], counts of
 *                               unique_consecutive with zeros kept),
 *   - by (expert, slot):        counts_k [E*P], pos_k [T*k],
 * where slot = level_to_precision(level) (moelab/policy.py:188-192) over P precisions.
 * n_kept [1] receives the number of kept pairs. level/skip may be NULL (all level 0 / none). */
int moeb200_dispatch(const int64_t* idx, const uint8_t* level, const uint8_t* skip, int32_t T, int32_t k,
                     int32_t E, int32_t P, int32_t* counts_e, int32_t* pos_e, int32_t* counts_k,
                     int32_t* pos_k, int32_t* n_kept, void* ws, size_t ws_bytes, void* stream);
size_t moeb200_dispatch_workspace(int32_t T, int32_t k, int32_t E, int32_t P);

/* ---- grouped expert products for one token --------------------------------------------------
 * Replaces grouped_ffn_int4 (moelab/kernels.py:834-872), grouped_ffn_int8 (kernels.py:747-769) and
 * grouped_ffn_float (kernels.py:875-891): out[H] += sum_e w[e] * down_e(silu(gate_e x) * up_e x)
 * for n experts sharing one layout. tab [n,4] (device) holds per expert the field addresses
 * [gate_up.q, gate_up.s, down.q, down.s] (float records: [gate_up, gate_up, down, down]), exactly
 * the pointer table of kernels.py:230-244. A row whose weight is 0 is a no-op (fixed-size tables,
 * kernels.py:903-905). x [H] and out [H] are act_type; accumulation is fp32. */
int moeb200_grouped_ffn(const moeb200_layout* layout, const int64_t* tab, const float* w, int32_t n,
                        const void* x, int32_t act_type, void* out, void* ws, size_t ws_bytes, void* stream);
size_t moeb200_grouped_ffn_workspace(const moeb200_layout* layout, int32_t n);

/* Workspace-free variant of moeb200_grouped_ffn (no counterpart in the reference).
 * For callers that cannot provide device scratch: a host binding the C ABI directly with no device
 * allocator of its own, or code that must not call cudaMalloc (it can synchronise the device, or the
 * GPU memory is already budgeted by another framework's allocator). The scratch is one static device
 * array of MOEB200_NOALLOC_SCRATCH_BYTES per GPU, held until the process exits; the call allocates
 * nothing. The first call on a device looks up that array's address with the device current, so make
 * it before any stream capture. Calls share the array: sequential calls are independent (what must
 * start at zero is cleared), calls that overlap on the GPU race. A call whose scratch would exceed
 * the array (moeb200_grouped_ffn_workspace(layout, n) > MOEB200_NOALLOC_SCRATCH_BYTES) returns
 * MOEB200_ERR_UNSUPPORTED without launching anything. */
#define MOEB200_NOALLOC_SCRATCH_BYTES (1u << 20)
int moeb200_grouped_ffn_noalloc(const moeb200_layout* layout, const int64_t* tab, const float* w, int32_t n,
                                const void* x, int32_t act_type, void* out, void* stream);
/* Companion of moeb200_grouped_ffn_noalloc (no counterpart in the reference). The static scratch
 * array of the current device starts with the same device status word as every workspace (see
 * moeb200_check_workspace); the workspace-free calls never clear it, so a bounded wait that gave up
 * or a bad index in any of them since the last check is kept. This call copies the word to *status
 * and clears it, synchronising the stream. The array's address is cached per device ordinal, which
 * assumes one context per device (the runtime's primary context). */
int moeb200_noalloc_check_status(int32_t* status, void* stream);

/* ---- the experts module ------------------------------------------------------------------------
 * Replaces OffloadedExperts.forward -> MoERuntime.run_layer for experts resident on this GPU
 * (moelab/runtime.py:522-770 with every request a VRAM hit; fullgraph.py:149-188 on device):
 * out[T,H] = sum over kept pairs (t,j) of w[t,j] * expert_{idx[t,j]}(x[t]) evaluated at the pair's
 * precision slot (level_to_precision of level[t,j]). out is overwritten (act_type).
 * level/skip may be NULL (every pair at slot 0). A pair whose expert has no resident record at its
 * slot is skipped and counted in miss [1] (fullgraph.py `flag`); miss may be NULL. */
int moeb200_experts_forward(const moeb200_expert_table* experts, const void* x, int32_t act_type, int32_t T,
                            const int64_t* idx, const float* w, int32_t k, const uint8_t* level,
                            const uint8_t* skip, void* out, int32_t* miss, void* ws, size_t ws_bytes,
                            void* stream);
size_t moeb200_experts_workspace(const moeb200_expert_table* experts, int32_t T, int32_t k);
/* ---- expert parallelism (no reference counterpart: moelab runs on one GPU) ---------------------
 * moeb200_experts_forward restricted to the experts [e_lo, e_hi) that this GPU owns: pairs routed to
 * other experts are dropped (not counted in miss), and the fp32 sums over the kept pairs are written
 * to part [T,H] (overwritten, not cast), so partial results of several GPUs can be added exactly.
 * Uses the workspace of moeb200_experts_workspace(experts, T, k). */
int moeb200_experts_forward_part(const moeb200_expert_table* experts, int32_t e_lo, int32_t e_hi, const void* x,
                                 int32_t act_type, int32_t T, const int64_t* idx, const float* w, int32_t k,
                                 const uint8_t* level, const uint8_t* skip, float* part, int32_t* miss, void* ws,
                                 size_t ws_bytes, void* stream);
/* Combine of expert-parallel partial sums: out[i] = act_type(sum over s = 0..G-1, in that order, of
 * parts[s*n + i]) (+ out[i] first when add != 0), i < n. act_type: F32, F16 or BF16. */
int moeb200_combine_parts(const float* parts, int32_t G, int64_t n, int32_t act_type, void* out, int32_t add,
                          void* stream);
/* Exchange rows: one token as [x: H act_type values | idx: k int64 | w: k float32 | level: k uint8 |
 * skip: k uint8 | zero padding to a multiple of 16 bytes] (moeb200_ep_row_bytes bytes), so one
 * collective or peer copy moves a rank's tokens with their routing. level/skip NULL on pack write
 * zeros; on unpack x, level and skip may be NULL (not written). x and rows 16-byte aligned. */
size_t moeb200_ep_row_bytes(int32_t H, int32_t k, int32_t act_type);
int moeb200_ep_pack(const void* x, const int64_t* idx, const float* w, const uint8_t* level, const uint8_t* skip,
                    int32_t T, int32_t H, int32_t k, int32_t act_type, void* rows, void* stream);
int moeb200_ep_unpack(const void* rows, int32_t n, int32_t H, int32_t k, int32_t act_type, void* x, int64_t* idx,
                      float* w, uint8_t* level, uint8_t* skip, void* stream);
/* ---- peer-memory exchange (expert parallelism without collectives) ------------------------------
 * Buffers a rank's peers map with CUDA IPC: moeb200_peer_alloc returns zeroed device memory and its
 * 64-byte IPC handle; a peer maps it with moeb200_peer_open (and unmaps with moeb200_peer_close).
 * A peer group describes, for every rank s < G, the device addresses (as mapped in this process) of
 * rank s's packed exchange rows [T, moeb200_ep_row_bytes], its fp32 partial sums [G*T, H] and its
 * flags int32 [2][G]; epoch is this rank's call counter and status its status word (device int32,
 * zero at setup). Per layer: moeb200_ep_pack into the own rows, moeb200_ep_signal(0), moeb200_ep_gather
 * (waits for every rank's rows, reads them over NVLink, unpacks to [G*T] arrays), the owned experts'
 * moeb200_experts_forward_part into the own partial sums, moeb200_ep_signal(1),
 * moeb200_ep_combine_peers (waits for every rank's partial sums, adds this rank's tokens' rows in
 * rank order, casts once). Waits are bounded: on timeout the status word is set. Every rank must run
 * the same sequence of calls with the same T. spin is the number of polls a wait makes before it
 * gives up (0 = 2^22, several seconds; each poll sleeps about 64 ns); a smaller budget makes a
 * missing peer show up in the status word sooner. */
typedef struct {
  int32_t G, rank, T, H, k;
  uint32_t spin;         /* polls per wait, 0 = default */
  const int64_t* rows;   /* [G] device array */
  const int64_t* parts;  /* [G] device array */
  const int64_t* flags;  /* [G] device array */
  int32_t* epoch;        /* [1] device */
  int32_t* status;       /* [1] device */
} moeb200_peer_group;
int moeb200_peer_alloc(size_t bytes, void** ptr, void* handle);
int moeb200_peer_open(const void* handle, void** ptr);
int moeb200_peer_close(void* ptr);
int moeb200_peer_free(void* ptr);
int moeb200_ep_signal(const moeb200_peer_group* group, int32_t which, void* stream);
int moeb200_ep_gather(const moeb200_peer_group* group, int32_t act_type, void* x, int64_t* idx, float* w,
                      uint8_t* level, uint8_t* skip, void* stream);
int moeb200_ep_combine_peers(const moeb200_peer_group* group, int32_t act_type, void* out, int32_t add, void* stream);

/* ---- dense int8 layers ------------------------------------------------------------------------
 * Replace moelab's QLinear (denseq.py:60-104), the non-expert nn.Linear layers quantised to int8
 * with one fp16 scale per group of gs input columns (quant.py `quantize(w, 8, gs)`):
 *   q [O, K] int8 (row-major), s [O, K/gs] fp16 bits.
 * moeb200_dense_int8_gemv replaces the one-token Triton kernel `_gemv8` (denseq.py:34-57) for up to 8
 * tokens: y[t, o] = act(sum_g s[o,g] * sum_{c in g} q[o,c] * x[t,c]) (fp32 accumulation), then
 * + bias[o] in the activation type when bias (act_type, [O]) is not NULL. x [T, K], y [T, O];
 * gs a multiple of 16 dividing K; q and x 16-byte aligned.
 * moeb200_dense_int8_dequant is the prefill half (denseq.py:94-100 + quant.py:191-205): w [O, K] =
 * act(q) * act(s) rounded once, the exact values of moelab's dequantize(q, s, 8, dtype). */
int moeb200_dense_int8_gemv(const int8_t* q, const uint16_t* s, int32_t O, int32_t K, int32_t gs, const void* x,
                            int32_t act_type, int32_t T, const void* bias, void* y, void* stream);
int moeb200_dense_int8_dequant(const int8_t* q, const uint16_t* s, int32_t O, int32_t K, int32_t gs,
                               int32_t act_type, void* w, void* stream);

/* ---- record quantiser -------------------------------------------------------------------------
 * moelab's quantize(w, bits, gs, method) (quant.py:104-127) on the device: w [O, K] (w_type F32, F16 or
 * BF16) -> q (bits 8: int8 [O, K]; bits 4: uint8 [O, K/2], +8, low nibble = even column) and fp16
 * scales s [O, K/gs]. method 0 = "absmax", 1 = "mse" (quant.py:64-93 scale search). fp32 arithmetic
 * with IEEE division; the mse error sums are added in numpy's pairwise order. gs <= 256 (even for
 * int4) dividing K. */
int moeb200_quantize(const void* w, int32_t w_type, int32_t O, int32_t K, int32_t bits, int32_t gs, int32_t method,
                     void* q, uint16_t* s, void* stream);

/* ---- shared expert ---------------------------------------------------------------------------
 * Replaces the shared-expert branch of Qwen3NextSparseMoeBlock.forward
 * (qwen3_next/modeling_qwen3_next.py:789-801), which runs beside the experts module:
 *   out[t] (+)= sigmoid(x[t] . wg) * down(silu(gate x[t]) * up x[t])   for t < T.
 * The shared MLP is one record of any store precision (gate_up = [gate_proj; up_proj], down =
 * down_proj; 256-byte aligned). wg [H] (act_type) is the shared_expert_gate weight: the logit is
 * accumulated in fp32 and rounded to act_type as F.linear returns it, the sigmoid is fp32.
 * add != 0 adds into out (after the routed experts), 0 overwrites it. */
int moeb200_shared_expert(const moeb200_layout* layout, const void* record, const void* wg, const void* x,
                          int32_t act_type, int32_t T, void* out, int32_t add, void* ws, size_t ws_bytes,
                          void* stream);
size_t moeb200_shared_expert_workspace(const moeb200_layout* layout, int32_t T);
/* Every workspace starts with a device status word that kernels set instead of hanging or
 * faulting (0 = OK, 1 = a bounded wait gave up, 2 = an expert index outside [0, E) reached
 * dispatch). This call copies it to *status and clears it; it is the one entry point that
 * synchronises the stream, so keep it out of captured graphs. */
int moeb200_check_workspace(void* ws, int32_t* status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MOEB200_H */
