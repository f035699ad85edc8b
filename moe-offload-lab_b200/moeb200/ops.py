"""torch-tensor wrappers of the C ABI: device pointers, the current stream and cached workspaces.

Every function here launches CUDA kernels of libmoeb200 on ``torch.cuda.current_stream()`` and
returns without synchronising. Inputs must already be CUDA tensors; nothing is computed on the CPU.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib
from .format import ACT_TYPE

_WS: dict[tuple[int, int], torch.Tensor] = {}
# Buffers replaced by a larger one. A CUDA graph captured while one of them was current keeps its
# address, so they stay allocated: replaying such a graph after a larger call grew the workspace
# must not touch freed memory. Growth at least doubles, so the retired buffers of a (device, slot)
# together are smaller than its current one.
_RETIRED: list[torch.Tensor] = []


def workspace(nbytes: int, device: torch.device, slot: int = 0) -> torch.Tensor:
    """A cached uint8 device buffer of at least nbytes (one per device and slot).

    Slots let callers that run concurrently keep separate scratch. The buffer only grows, and a
    buffer that was replaced stays allocated (see release_workspaces), so graphs captured with it
    stay valid; replays of graphs that share a slot must not overlap on the GPU.
    """
    dev = torch.device(device)
    key = (dev.index if dev.index is not None else torch.cuda.current_device(), slot)
    buf = _WS.get(key)
    if buf is None or buf.numel() < nbytes:
        if buf is not None:
            _RETIRED.append(buf)
        grow = 2 * buf.numel() if buf is not None else 0
        buf = torch.zeros(max(nbytes, grow, 1 << 16), dtype=torch.uint8, device=dev)  # status word 0
        _WS[key] = buf
    return buf


def release_workspaces() -> None:
    """Free the replaced workspaces. Only safe once no captured graph that used them is replayed."""
    _RETIRED.clear()


def _stream(device=None) -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t: torch.Tensor | None) -> C.c_void_p:
    return C.c_void_p(t.data_ptr() if t is not None else 0)


def _need_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("moeb200 kernels take CUDA tensors only (there is no CPU path)")


def _act(dtype: torch.dtype) -> int:
    if dtype not in ACT_TYPE:
        raise ValueError(f"unsupported activation dtype {dtype}")
    return ACT_TYPE[dtype]


@dataclass
class PolicySpec:
    """Precision rule of the experts module (moelab/policy.py:20-58 PrecisionPolicy, plus the
    threshold rule of the build's configs). mode: "hi", "lo", "hobbit" or "threshold"."""

    mode: str = "hobbit"
    t1: float = 0.6
    t_mid: float | None = None
    t2: float | None = None
    thr: float = 0.1
    protect_layers: frozenset = frozenset()
    # per-expert vote of the reference's multi-token path (moelab/policy.py:148-154; its default
    # hi_vote is 0.5): None = every pair keeps its own level
    hi_vote: float | None = None

    def to_c(self, layer: int | None = None) -> _lib.Policy:
        mode = self.mode
        if layer is not None and layer in self.protect_layers:
            mode = "hi"
        p = _lib.Policy()
        p.mode = {"hi": 0, "lo": 1, "hobbit": 2, "threshold": 3}[mode]
        p.t1 = self.t1
        p.t_mid = -1.0 if self.t_mid is None else self.t_mid
        p.t2 = -1.0 if self.t2 is None else self.t2
        p.thr = self.thr
        return p


def router(h: torch.Tensor, wr: torch.Tensor, k: int, renorm: bool, bias: torch.Tensor | None = None,
           policy: _lib.Policy | None = None, want_probs: bool = True, out: dict | None = None,
           logits: torch.Tensor | None = None, shared_level: int | None = None):
    """Fused router: (probs [T,E] f32 | None, w [T,k] f32, idx [T,k] i64, level [T,k] u8 | None,
    skip [T,k] u8 | None).

    shared_level (Qwen3-Next shared expert folded in): wr holds E + 1 rows, the last one the shared
    expert's gate; w / idx / level / skip gain a (k+1)-th column per token = (expert E,
    sigmoid(x . wg), shared_level, not skipped)."""
    _need_cuda(h, wr, bias)
    T, H = h.shape
    sh = shared_level is not None
    E = wr.shape[0] - (1 if sh else 0)
    kk = k + (1 if sh else 0)
    dev = h.device
    o = out or {}
    probs = o.get("probs") if want_probs else None
    if want_probs and probs is None:
        probs = torch.empty(T, E, dtype=torch.float32, device=dev)
    w = o.get("w")
    if w is None:
        w = torch.empty(T, kk, dtype=torch.float32, device=dev)
    idx = o.get("idx")
    if idx is None:
        idx = torch.empty(T, kk, dtype=torch.int64, device=dev)
    level = skip = None
    if policy is not None:
        level = o.get("level")
        if level is None:
            level = torch.empty(T, kk, dtype=torch.uint8, device=dev)
        skip = o.get("skip")
        if skip is None:
            skip = torch.empty(T, kk, dtype=torch.uint8, device=dev)
    for name, t in (("w", w), ("idx", idx), ("level", level), ("skip", skip)):
        if t is not None and (tuple(t.shape) != (T, kk) or not t.is_contiguous()):
            raise ValueError(f"{name} must be a contiguous [{T}, {kk}] tensor")
    L = _lib.lib()
    nbytes = L.moeb200_router_workspace(T, E + (1 if sh else 0))
    ws = workspace(nbytes, dev, slot=1)
    pol = C.byref(policy) if policy is not None else None
    if sh:
        _lib.check(L.moeb200_router_shared(_ptr(h), _ptr(wr), _ptr(bias), _act(h.dtype), T, H, E, k,
                                           int(bool(renorm)), int(shared_level), _ptr(probs), _ptr(w), _ptr(idx),
                                           _ptr(logits), pol, _ptr(level), _ptr(skip), _ptr(ws), ws.numel(),
                                           _stream(dev)))
    else:
        _lib.check(L.moeb200_router(_ptr(h), _ptr(wr), _ptr(bias), _act(h.dtype), T, H, E, k, int(bool(renorm)),
                                    _ptr(probs), _ptr(w), _ptr(idx), _ptr(logits), pol,
                                    _ptr(level), _ptr(skip), _ptr(ws), ws.numel(), _stream(dev)))
    return probs, w, idx, level, skip


def levels(w: torch.Tensor, policy: _lib.Policy, level: torch.Tensor | None = None,
           skip: torch.Tensor | None = None):
    _need_cuda(w)
    T, k = w.shape
    if level is None:
        level = torch.empty(T, k, dtype=torch.uint8, device=w.device)
    if skip is None:
        skip = torch.empty(T, k, dtype=torch.uint8, device=w.device)
    _lib.check(_lib.lib().moeb200_levels(_ptr(w), T, k, C.byref(policy), _ptr(level), _ptr(skip),
                                         _stream(w.device)))
    return level, skip


def levels_vote(idx: torch.Tensor, level: torch.Tensor, skip: torch.Tensor | None, E: int, hi_vote: float) -> torch.Tensor:
    """Rewrite level [T,k] in place with each expert's vote over its kept pairs (moelab/policy.py:148-154)."""
    _need_cuda(idx, level, skip)
    T, k = idx.shape
    if idx.dtype != torch.int64 or level.dtype != torch.uint8 or not (idx.is_contiguous() and level.is_contiguous()):
        raise ValueError("idx must be contiguous int64 and level contiguous uint8")
    _lib.check(_lib.lib().moeb200_levels_vote(_ptr(idx), _ptr(level), _ptr(skip), T, k, E, float(hi_vote),
                                              _stream(idx.device)))
    return level


def dispatch(idx: torch.Tensor, level: torch.Tensor | None, skip: torch.Tensor | None, E: int, P: int):
    """Stable dispatch: dict(counts_e [E], pos_e [T*k], counts_k [E*P], pos_k [T*k], n_kept [1])."""
    _need_cuda(idx, level, skip)
    T, k = idx.shape
    dev = idx.device
    n = T * k
    counts_e = torch.empty(E, dtype=torch.int32, device=dev)
    counts_k = torch.empty(E * P, dtype=torch.int32, device=dev)
    pos_e = torch.full((n,), -1, dtype=torch.int32, device=dev)
    pos_k = torch.full((n,), -1, dtype=torch.int32, device=dev)
    n_kept = torch.empty(1, dtype=torch.int32, device=dev)
    L = _lib.lib()
    ws = workspace(L.moeb200_dispatch_workspace(T, k, E, P), dev, slot=2)
    _lib.check(L.moeb200_dispatch(_ptr(idx.contiguous()), _ptr(level), _ptr(skip), T, k, E, P, _ptr(counts_e),
                                  _ptr(pos_e), _ptr(counts_k), _ptr(pos_k), _ptr(n_kept), _ptr(ws), ws.numel(),
                                  _stream(dev)))
    return {"counts_e": counts_e, "pos_e": pos_e, "counts_k": counts_k, "pos_k": pos_k, "n_kept": n_kept}


def grouped_ffn_table(layout_c: _lib.Layout, tab: torch.Tensor, w: torch.Tensor, x_row: torch.Tensor,
                      out: torch.Tensor, ws: torch.Tensor | None = None) -> None:
    """out[H] += sum_e w[e] * expert_e(x) with a device pointer table tab [n, 4] (int64)."""
    _need_cuda(tab, w, x_row, out)
    n = tab.shape[0]
    L = _lib.lib()
    nbytes = L.moeb200_grouped_ffn_workspace(C.byref(layout_c), n)
    if ws is None:
        ws = workspace(nbytes, x_row.device, slot=3)
    elif ws.numel() < nbytes:
        raise ValueError("workspace too small")
    _lib.check(L.moeb200_grouped_ffn(C.byref(layout_c), _ptr(tab), _ptr(w), n, _ptr(x_row), _act(x_row.dtype),
                                     _ptr(out), _ptr(ws), ws.numel(), _stream(x_row.device)))


def experts_forward(table: _lib.ExpertTable, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor,
                    level: torch.Tensor | None, skip: torch.Tensor | None, out: torch.Tensor | None = None,
                    miss: torch.Tensor | None = None, ws: torch.Tensor | None = None) -> torch.Tensor:
    """out[T,H] = sum over kept pairs of w * expert(x) at each pair's precision slot."""
    _need_cuda(x, idx, w, level, skip)
    T = x.shape[0]
    k = idx.shape[1]
    if out is None:
        out = torch.empty_like(x)
    L = _lib.lib()
    nbytes = L.moeb200_experts_workspace(C.byref(table), T, k)
    if ws is None:
        ws = workspace(nbytes, x.device, slot=0)
    elif ws.numel() < nbytes:
        raise ValueError("workspace too small")
    _lib.check(L.moeb200_experts_forward(C.byref(table), _ptr(x), _act(x.dtype), T, _ptr(idx), _ptr(w), k,
                                         _ptr(level), _ptr(skip), _ptr(out), _ptr(miss), _ptr(ws), ws.numel(),
                                         _stream(x.device)))
    return out


def experts_forward_part(table: _lib.ExpertTable, e_lo: int, e_hi: int, x: torch.Tensor, idx: torch.Tensor,
                         w: torch.Tensor, level: torch.Tensor | None, skip: torch.Tensor | None,
                         part: torch.Tensor | None = None, miss: torch.Tensor | None = None,
                         ws: torch.Tensor | None = None) -> torch.Tensor:
    """part[T,H] fp32 = sum over the kept pairs routed to experts [e_lo, e_hi) of w * expert(x)."""
    _need_cuda(x, idx, w, level, skip)
    T = x.shape[0]
    k = idx.shape[1]
    if part is None:
        part = torch.empty(T, x.shape[1], dtype=torch.float32, device=x.device)
    if part.dtype != torch.float32 or part.shape != (T, x.shape[1]) or not part.is_contiguous():
        raise ValueError("part must be a contiguous float32 [T, H] tensor")
    L = _lib.lib()
    nbytes = L.moeb200_experts_workspace(C.byref(table), T, k)
    if ws is None:
        ws = workspace(nbytes, x.device, slot=0)
    elif ws.numel() < nbytes:
        raise ValueError("workspace too small")
    _lib.check(L.moeb200_experts_forward_part(C.byref(table), e_lo, e_hi, _ptr(x), _act(x.dtype), T, _ptr(idx),
                                              _ptr(w), k, _ptr(level), _ptr(skip), _ptr(part), _ptr(miss), _ptr(ws),
                                              ws.numel(), _stream(x.device)))
    return part


def combine_parts(parts: torch.Tensor, out: torch.Tensor, add: bool = False) -> torch.Tensor:
    """out = cast(sum over parts[0..G-1]) in that order (+ out when add); parts fp32 [G, *out.shape]."""
    _need_cuda(parts, out)
    if parts.dtype != torch.float32 or not parts.is_contiguous() or parts.shape[1:] != out.shape:
        raise ValueError("parts must be contiguous float32 [G, *out.shape]")
    if not out.is_contiguous():
        raise ValueError("out must be contiguous")
    _lib.check(_lib.lib().moeb200_combine_parts(_ptr(parts), parts.shape[0], out.numel(), _act(out.dtype), _ptr(out),
                                                int(add), _stream(out.device)))
    return out


def ep_row_bytes(H: int, k: int, dtype: torch.dtype) -> int:
    """Bytes of one exchange row (token hidden row + its routing) for expert parallelism."""
    return int(_lib.lib().moeb200_ep_row_bytes(H, k, _act(dtype)))


def ep_pack(x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, level: torch.Tensor | None,
            skip: torch.Tensor | None, rows: torch.Tensor | None = None) -> torch.Tensor:
    """rows [T, ep_row_bytes] uint8 = each token's hidden row followed by its routing."""
    _need_cuda(x, idx, w, level, skip)
    T, H = x.shape
    k = idx.shape[1]
    rb = ep_row_bytes(H, k, x.dtype)
    if rows is None:
        rows = torch.empty(T, rb, dtype=torch.uint8, device=x.device)
    if rows.shape != (T, rb) or rows.dtype != torch.uint8 or not rows.is_contiguous():
        raise ValueError(f"rows must be contiguous uint8 [{T}, {rb}]")
    _lib.check(_lib.lib().moeb200_ep_pack(_ptr(x), _ptr(idx), _ptr(w), _ptr(level), _ptr(skip), T, H, k,
                                          _act(x.dtype), _ptr(rows), _stream(x.device)))
    return rows


def ep_unpack(rows: torch.Tensor, H: int, k: int, dtype: torch.dtype, x: torch.Tensor, idx: torch.Tensor,
              w: torch.Tensor, level: torch.Tensor | None, skip: torch.Tensor | None) -> None:
    """Split exchange rows [n, ep_row_bytes] back into x [n,H], idx/w/level/skip [n,k]."""
    _need_cuda(rows, x, idx, w, level, skip)
    n = rows.shape[0]
    if rows.shape[1] != ep_row_bytes(H, k, dtype) or not rows.is_contiguous():
        raise ValueError("rows do not match (H, k, dtype)")
    _lib.check(_lib.lib().moeb200_ep_unpack(_ptr(rows), n, H, k, _act(dtype), _ptr(x), _ptr(idx), _ptr(w),
                                            _ptr(level), _ptr(skip), _stream(rows.device)))


def shared_expert(layout_c: _lib.Layout, record: torch.Tensor, wg: torch.Tensor, x: torch.Tensor,
                  out: torch.Tensor | None = None, add: bool = False, ws: torch.Tensor | None = None) -> torch.Tensor:
    """out (+)= sigmoid(x . wg) * SwiGLU_shared(x) (Qwen3-Next shared expert; one record)."""
    _need_cuda(record, wg, x, out)
    T = x.shape[0]
    if out is None:
        out = torch.empty_like(x)
        add = False
    L = _lib.lib()
    nbytes = L.moeb200_shared_expert_workspace(C.byref(layout_c), T)
    if ws is None:
        ws = workspace(nbytes, x.device, slot=4)
    elif ws.numel() < nbytes:
        raise ValueError("workspace too small")
    _lib.check(L.moeb200_shared_expert(C.byref(layout_c), _ptr(record), _ptr(wg), _ptr(x), _act(x.dtype), T, _ptr(out),
                                       int(add), _ptr(ws), ws.numel(), _stream(x.device)))
    return out


def set_path(path: str) -> None:
    """Expert-product path for this thread's next experts_forward calls: "auto", "gemv", "gemm", "decode"
    (the fused one-launch decode kernel) or "ws" (the warp-streamed grouped GEMV)."""
    _lib.check(_lib.lib().moeb200_set_path({"auto": 0, "gemv": 1, "gemm": 2, "decode": 3, "ws": 4}[path]))


def set_item_tokens(nt: int) -> None:
    """Pairs per grouped-GEMV work item for this thread's next experts_forward calls (0 = auto, 8, 16)."""
    _lib.check(_lib.lib().moeb200_set_item_tokens(nt))


def check_workspace(ws: torch.Tensor) -> int:
    """Device status word of a workspace (0 = OK); synchronises the current stream."""
    st = C.c_int32(0)
    _lib.check(_lib.lib().moeb200_check_workspace(_ptr(ws), C.byref(st), _stream(ws.device)))
    return st.value


def dense_int8_gemv(q: torch.Tensor, s: torch.Tensor, group_size: int, x: torch.Tensor,
                    bias: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """y [T, O] = x [T, K] @ dequant(q, s).T (+ bias) for T <= 8 tokens; q int8 [O, K], s fp16 [O, K/gs]."""
    _need_cuda(q, s, x, bias, out)
    O, K = q.shape
    T = x.shape[0]
    if q.dtype != torch.int8 or s.dtype != torch.float16 or s.shape != (O, K // group_size):
        raise ValueError("q must be int8 [O, K] and s float16 [O, K/gs]")
    if not (q.is_contiguous() and s.is_contiguous() and x.is_contiguous()) or x.shape[1] != K:
        raise ValueError("q, s and x [T, K] must be contiguous")
    if bias is not None and (bias.dtype != x.dtype or bias.shape != (O,) or not bias.is_contiguous()):
        raise ValueError("bias must be contiguous [O] in the activation dtype")
    if out is None:
        out = torch.empty(T, O, dtype=x.dtype, device=x.device)
    _lib.check(_lib.lib().moeb200_dense_int8_gemv(_ptr(q), _ptr(s), O, K, group_size, _ptr(x), _act(x.dtype), T,
                                                  _ptr(bias), _ptr(out), _stream(x.device)))
    return out


def dense_int8_dequant(q: torch.Tensor, s: torch.Tensor, group_size: int, dtype: torch.dtype,
                       out: torch.Tensor | None = None) -> torch.Tensor:
    """w [O, K] in dtype = the exact values of moelab's dequantize(q, s, 8, dtype)."""
    _need_cuda(q, s, out)
    O, K = q.shape
    if out is None:
        out = torch.empty(O, K, dtype=dtype, device=q.device)
    if not (q.is_contiguous() and s.is_contiguous() and out.is_contiguous()) or out.shape != (O, K):
        raise ValueError("q, s and out must be contiguous, out [O, K]")
    _lib.check(_lib.lib().moeb200_dense_int8_dequant(_ptr(q), _ptr(s), O, K, group_size, _act(out.dtype), _ptr(out),
                                                     _stream(q.device)))
    return out


def quantize(w: torch.Tensor, bits: int, group_size: int, method: str = "absmax") -> tuple[torch.Tensor, torch.Tensor]:
    """moelab's quantize(w, bits, gs, method) on the device: (q, fp16 scales [O, K/gs]); q is int8 [O, K]
    (bits 8) or uint8 [O, K/2] (bits 4, two values per byte)."""
    _need_cuda(w)
    if w.dim() != 2 or not w.is_contiguous():
        raise ValueError("w must be a contiguous [O, K] matrix")
    O, K = w.shape
    wt = {torch.float32: _lib.F32, torch.float16: _lib.F16, torch.bfloat16: _lib.BF16}.get(w.dtype)
    if wt is None:
        raise ValueError("w must be float32, float16 or bfloat16")
    m = {"absmax": 0, "mse": 1}[method]
    q = torch.empty(O, K if bits == 8 else K // 2, dtype=torch.int8 if bits == 8 else torch.uint8, device=w.device)
    s = torch.empty(O, K // group_size, dtype=torch.float16, device=w.device)
    _lib.check(_lib.lib().moeb200_quantize(_ptr(w), wt, O, K, bits, group_size, m, _ptr(q), _ptr(s),
                                           _stream(w.device)))
    return q, s
