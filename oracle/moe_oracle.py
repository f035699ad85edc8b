"""CPU oracle for the MoE-layer hot path -- TEST INFRASTRUCTURE ONLY.

This module is a plain numpy restatement of the reference's algorithm for the MoE layer of
moelab (VictorCourtois135/moe-offload-lab). It is the checker for the CUDA path: only tests,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py``
may import it. The product path never imports, calls or falls back to it.

Parity pins (tests/test_oracle_golden.py): every function below is checked against golden
vectors produced by the reference itself (tests/golden/make_golden.py imports moelab and the
installed transformers in the build container), and against the known answers held by the
reference's own tests (tests/test_units.py, tests/test_kernels.py).

Reference citations are ``path:line`` inside the moelab project.
"""

from __future__ import annotations

import math

import numpy as np

# ---------------------------------------------------------------------------------------------
# Format: quantiser and expert records (moelab/quant.py, moelab/store.py)
# ---------------------------------------------------------------------------------------------

ALIGN = 4096          # record alignment, moelab/store.py:36
FIELD_ALIGN = 64      # field alignment inside a record, moelab/store.py:37
QMAX = {8: 127, 4: 7}     # moelab/quant.py:43
QMIN = {8: -127, 4: -8}   # moelab/quant.py:44
_GRID = [1.0 - 0.02 * i for i in range(16)]  # scale search grid 1.00 .. 0.70, moelab/quant.py:46

PRECISIONS = {  # moelab/store.py:39-45
    "fp32": ("float", "float32"),
    "fp16": ("float", "float16"),
    "bf16": ("float", "bfloat16"),
    "int8": ("int", 8),
    "int4": ("int", 4),
}
ELEM = {"float32": 4, "float16": 2, "bfloat16": 2, "int8": 1, "uint8": 1}


def _align(n: int, a: int) -> int:
    return (n + a - 1) // a * a


def pick_group_size(in_features: int, preferred: int = 64) -> int:
    """Largest even group size <= preferred dividing in_features (moelab/quant.py:49-54)."""
    for gs in range(min(preferred, in_features), 1, -1):
        if in_features % gs == 0 and gs % 2 == 0:
            return gs
    raise ValueError(f"no even group size divides {in_features}")


def record_layout(prec: str, hidden: int, inter: int, group_size: int = 64, scale: str | None = None) -> dict:
    """Field table of one expert record (moelab/store.py:76-115).

    gate_up is [2*inter, hidden] (gate rows then up rows), down is [hidden, inter]. Integer
    precisions store ``<name>.q`` then ``<name>.s`` (fp16 scale per group along the input dim).
    Every field starts on a 64-byte boundary; the record is padded to 4096 bytes.
    """
    kind, arg = PRECISIONS[prec]
    if kind == "int" and scale is None:
        scale = "mse" if arg == 4 else "absmax"
    mats = {"gate_up": (2 * inter, hidden), "down": (hidden, inter)}
    raw = []
    groups = {}
    if kind == "float":
        for name, shape in mats.items():
            raw.append((name, shape, arg))
    else:
        for name, (o, i) in mats.items():
            gs = pick_group_size(i, group_size)
            groups[name] = gs
            raw.append((f"{name}.q", (o, i) if arg == 8 else (o, i // 2), "int8" if arg == 8 else "uint8"))
            raw.append((f"{name}.s", (o, i // gs), "float16"))
    fields, off = [], 0
    for name, shape, dt in raw:
        fields.append([name, list(shape), dt, off])
        n = ELEM[dt]
        for s in shape:
            n *= s
        off = _align(off + n, FIELD_ALIGN)
    lay = {"precision": prec, "fields": fields, "record_bytes": _align(off, ALIGN), "group_sizes": groups}
    if kind == "int":
        lay["scale"] = scale
    return lay


def _f16(a) -> np.ndarray:
    return np.asarray(a, dtype=np.float32).astype(np.float16)


def _safe(s32: np.ndarray) -> np.ndarray:
    """Scale rounded to fp16 and never zero (moelab/quant.py:57-61)."""
    s16 = s32.astype(np.float16)
    return np.where(s16 == 0, np.float16(1e-7), s16)


def choose_scales(wf: np.ndarray, bits: int, method: str = "absmax") -> np.ndarray:
    """fp16 scale of each group (last axis = one group), shape (..., 1) (moelab/quant.py:64-93).

    "absmax": max|w| / qmax. "mse": candidates max|w|/qmax and (int4 only) the signed max / -8,
    each times 1.00, 0.98 .. 0.70; keep the one with the least squared error, first one on ties.
    All arithmetic is float32, as in the reference.
    """
    qmin, qmax = QMIN[bits], QMAX[bits]
    wf = wf.astype(np.float32)
    absmax = np.abs(wf).max(axis=-1, keepdims=True)
    if method == "absmax":
        return _safe(np.maximum(absmax / np.float32(qmax), np.float32(1e-7)))
    bases = [absmax / np.float32(qmax)]
    if qmin == -qmax - 1:
        am = np.abs(wf).argmax(axis=-1)[..., None]
        mx = np.take_along_axis(wf, am, axis=-1)
        bases.append(mx / np.float32(qmin))
    best_s = best_e = None
    for b in bases:
        for f in _GRID:
            s = _safe(b * np.float32(f))
            sf = s.astype(np.float32)
            q = np.clip(np.round(wf / sf), qmin, qmax)
            err = ((q * sf - wf) ** 2).sum(axis=-1, keepdims=True, dtype=np.float32)
            if best_s is None:
                best_s, best_e = s, err
            else:
                better = err < best_e
                best_s = np.where(better, s, best_s)
                best_e = np.where(better, err, best_e)
    return best_s


def pack(q: np.ndarray, bits: int) -> np.ndarray:
    """Integers (out, in) -> stored form (moelab/quant.py:96-101).

    int8: one signed byte per value. int4: two values per byte, stored +8 in [0, 15];
    the low nibble is the even column, the high nibble the odd column.
    """
    if bits == 8:
        return q.astype(np.int8)
    u = (q + 8).astype(np.uint8)
    return (u[:, 0::2] | (u[:, 1::2] << 4)).astype(np.uint8)


def quantize(w: np.ndarray, bits: int, group_size: int, method: str = "absmax"):
    """(out, in) float -> (packed q, fp16 scales [out, in/gs]) (moelab/quant.py:104-127)."""
    out_f, in_f = w.shape
    if in_f % group_size:
        raise ValueError("in_features not divisible by group_size")
    wf = w.astype(np.float32).reshape(out_f, in_f // group_size, group_size)
    s = choose_scales(wf, bits, method)
    q = np.clip(np.round(wf / s.astype(np.float32)), QMIN[bits], QMAX[bits]).astype(np.int16)
    return pack(q.reshape(out_f, in_f), bits), s.reshape(out_f, in_f // group_size)


def dequantize(q: np.ndarray, scales: np.ndarray, bits: int) -> np.ndarray:
    """Stored integers + fp16 scales -> float32 weights (moelab/quant.py:191-205, fp32 target).

    int4 value = nibble - 8 (low nibble = even column); int8 value = q. Product in fp32 is
    exact (at most 4 or 8 bits times an 11-bit fp16 significand).
    """
    out_f = q.shape[0]
    if bits == 8:
        vals = q.astype(np.float32)
    else:
        lo = (q & 0x0F).astype(np.float32)
        hi = (q >> 4).astype(np.float32)
        vals = np.stack((lo, hi), axis=-1).reshape(out_f, q.shape[1] * 2) - np.float32(8)
    in_f = vals.shape[1]
    gs = in_f // scales.shape[1]
    return (vals.reshape(out_f, in_f // gs, gs) * scales.astype(np.float32)[..., None]).reshape(out_f, in_f)


def _np_dtype(dt: str):
    if dt == "bfloat16":
        return None
    return {"float32": np.float32, "float16": np.float16, "int8": np.int8, "uint8": np.uint8}[dt]


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns (uint16), round to nearest even (NaN kept quiet)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    r = ((u >> 16) & 1) + np.uint32(0x7FFF)
    out = ((u + r) >> 16).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        out = np.where(nan, np.uint16(0x7FC0), out)
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_to(a: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to fp16 / bf16 / fp32 and return them as float32."""
    a = np.asarray(a, dtype=np.float32)
    if dtype == "float16":
        return a.astype(np.float16).astype(np.float32)
    if dtype == "bfloat16":
        return bf16_bits_to_f32(f32_to_bf16_bits(a))
    return a


def encode_record(layout: dict, gate_up: np.ndarray, down: np.ndarray) -> np.ndarray:
    """Bytes of one record from float32 weights (moelab/store.py:122-150)."""
    kind, arg = PRECISIONS[layout["precision"]]
    buf = np.zeros(layout["record_bytes"], dtype=np.uint8)
    tensors = {}
    if kind == "float":
        for name, w in (("gate_up", gate_up), ("down", down)):
            if arg == "bfloat16":
                tensors[name] = f32_to_bf16_bits(w)
            else:
                tensors[name] = np.asarray(w, dtype=np.float32).astype(_np_dtype(arg))
    else:
        method = layout.get("scale") or "absmax"
        for name, w in (("gate_up", gate_up), ("down", down)):
            q, s = quantize(np.asarray(w, dtype=np.float32), arg, layout["group_sizes"][name],
                            "absmax" if method == "gptq" else method)
            tensors[f"{name}.q"], tensors[f"{name}.s"] = q, s
    for name, shape, dt, off in layout["fields"]:
        t = np.ascontiguousarray(tensors[name])
        assert tuple(t.shape) == tuple(shape), (name, t.shape, shape)
        raw = t.view(np.uint8).reshape(-1)
        buf[off:off + raw.size] = raw
    return buf


def views(layout: dict, blob: np.ndarray) -> dict:
    """Typed zero-copy views into one record (moelab/store.py:153-161). bf16 fields are uint16 bits."""
    out = {}
    for name, shape, dt, off in layout["fields"]:
        n = ELEM[dt]
        for s in shape:
            n *= s
        part = blob[off:off + n]
        if dt == "bfloat16":
            part = part.view(np.uint16)
        elif dt != "uint8":
            part = part.view(_np_dtype(dt))
        out[name] = part.reshape(shape)
    return out


def materialize_f32(layout: dict, blob: np.ndarray):
    """Record -> (gate_up, down) in float32 (moelab/store.py:164-174 with dtype=float32)."""
    v = views(layout, blob)
    kind, arg = PRECISIONS[layout["precision"]]
    if kind == "float":
        if arg == "bfloat16":
            return bf16_bits_to_f32(v["gate_up"]), bf16_bits_to_f32(v["down"])
        return v["gate_up"].astype(np.float32), v["down"].astype(np.float32)
    return dequantize(v["gate_up.q"], v["gate_up.s"], arg), dequantize(v["down.q"], v["down.s"], arg)


# ---------------------------------------------------------------------------------------------
# Router (installed transformers: olmoe/modeling_olmoe.py:350-359, qwen3_moe 254-272,
# qwen3_next 761-779; the router is the unchanged `gate` of the MoE block, moelab/loader.py:222)
# ---------------------------------------------------------------------------------------------

def _round_f64_to(a: np.ndarray, dtype: str) -> np.ndarray:
    """Round float64 values directly to fp16 / bf16 / fp32 (single rounding)."""
    if dtype == "float16":
        return a.astype(np.float16).astype(np.float32)
    if dtype == "float32":
        return a.astype(np.float32)
    # bf16: round the float64 to 8 significant bits, ties to even, in one step.
    m, e = np.frexp(a)
    r = np.ldexp(np.round(np.ldexp(m, 8)), e - 8)
    return r.astype(np.float32)


def router_logits_exact(h: np.ndarray, wr: np.ndarray, dtype: str) -> tuple[np.ndarray, np.ndarray]:
    """(rounded logits as float32, exact float64 logits)."""
    exact = np.asarray(h, dtype=np.float64) @ np.asarray(wr, dtype=np.float64).T
    return _round_f64_to(exact, dtype), exact


def topk_lower_index(vals: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest values per row, descending; equal values -> lower index first
    (the tie order fixed for the build; torch.topk leaves it unspecified)."""
    E = vals.shape[1]
    order = np.lexsort((np.broadcast_to(np.arange(E), vals.shape), -vals.astype(np.float64)), axis=-1)
    return order[:, :k].astype(np.int64)


def softmax_f32(logits: np.ndarray) -> np.ndarray:
    """softmax(dtype=float) over the expert axis: exp(l - max) / sum, in float32."""
    l = np.asarray(logits, dtype=np.float32)
    e = np.exp(l - l.max(axis=-1, keepdims=True))
    return (e / e.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)


def router(h: np.ndarray, wr: np.ndarray, k: int, renorm: bool, dtype: str, bias: np.ndarray | None = None):
    """TopK router: logits in the model dtype (+ optional per-expert bias in float32, the
    synthetic skew of the build's configs), softmax in fp32, top-k, optional renormalisation.
    Returns (probs [T,E] f32, weights [T,k] f32, idx [T,k] int64, logits [T,E] f32)."""
    logits, _ = router_logits_exact(h, wr, dtype)
    if bias is not None:
        logits = (logits + np.asarray(bias, dtype=np.float32)[None, :]).astype(np.float32)
    probs = softmax_f32(logits)
    idx = topk_lower_index(logits, k)
    w = np.take_along_axis(probs, idx, axis=-1)
    if renorm:
        w = (w / w.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)
    return probs, w.astype(np.float32), idx, logits


def topk_from_logits(logits: np.ndarray, k: int, renorm: bool):
    """The router's post-GEMV part on given (already rounded, biased) logits."""
    probs = softmax_f32(logits)
    idx = topk_lower_index(logits, k)
    w = np.take_along_axis(probs, idx, axis=-1)
    if renorm:
        w = (w / w.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)
    return probs, w.astype(np.float32), idx


# ---------------------------------------------------------------------------------------------
# Precision mask (moelab/policy.py)
# ---------------------------------------------------------------------------------------------

def unimportance(w: np.ndarray) -> np.ndarray:
    """HOBBIT score s [T,k] (moelab/policy.py:77-87): normalise the k weights, sort descending
    (stable), s = cumulative normalised mass of the better-ranked experts. float32, summed in
    rank order."""
    w = np.asarray(w, dtype=np.float32)
    T, k = w.shape
    s = np.zeros((T, k), dtype=np.float32)
    for t in range(T):
        tot = np.float32(0)
        for j in range(k):
            tot = np.float32(tot + w[t, j])
        tot = max(tot, np.float32(1e-12))
        wn = (w[t] / tot).astype(np.float32)
        order = sorted(range(k), key=lambda j: -float(wn[j]))
        acc = np.float32(0)
        for j in order:
            s[t, j] = acc
            acc = np.float32(acc + wn[j])
    return s


MODE_HI, MODE_LO, MODE_HOBBIT = 0, 1, 2


def hobbit_levels(w: np.ndarray, mode: int = MODE_HOBBIT, t1: float = 0.6, t_mid: float | None = None,
                  t2: float | None = None):
    """(level [T,k] uint8 in {0,1,2}, skip [T,k] bool) (moelab/policy.py:110-123, 125-137).

    level 0 if s <= t1 + 1e-6; 1 if t_mid is set and s <= t_mid + 1e-6; else 2.
    skip if t2 is set, s > t2 + 1e-6 and level != 0. Modes "hi"/"lo" (and protected layers,
    which the caller maps to "hi") fix every level to 0 / 2.
    """
    w = np.asarray(w, dtype=np.float32)
    T, k = w.shape
    if mode == MODE_HI:
        return np.zeros((T, k), np.uint8), np.zeros((T, k), bool)
    if mode == MODE_LO:
        return np.full((T, k), 2, np.uint8), np.zeros((T, k), bool)
    s = unimportance(w)
    lvl = np.full((T, k), 2, np.uint8)
    if t_mid is not None:
        lvl[s <= np.float32(t_mid + 1e-6)] = 1
    lvl[s <= np.float32(t1 + 1e-6)] = 0
    skip = (s > np.float32(t2 + 1e-6)) & (lvl != 0) if t2 is not None else np.zeros((T, k), bool)
    return lvl, skip


def threshold_levels(w: np.ndarray, thr: float):
    """Rule of the build's configs 1 and 4: level 0 (hi precision) if the pair's router
    probability >= thr, else level 2 (lowest precision). No pair is skipped."""
    w = np.asarray(w, dtype=np.float32)
    return np.where(w >= np.float32(thr), 0, 2).astype(np.uint8), np.zeros(w.shape, bool)


def expert_vote(idx: np.ndarray, level: np.ndarray, skip: np.ndarray | None, E: int, hi_vote: float = 0.5):
    """Per-expert precision vote of the reference's T > 1 path (moelab/policy.py:148-154
    `expert_level`, applied per expert in moelab/runtime.py:476-488 `_decide_general`).

    Over the kept (not skipped) pairs of expert e (n of them), the expert's level is the most
    precise level L in (0, 1) with #(pair levels <= L) >= (hi_vote - 1e-9) * n, else 2; the
    comparison is the reference's Python (double) arithmetic. Returns (vote [E] int8, -1 where the
    expert has no kept pair; levels [T, k] uint8 with every kept pair set to its expert's vote,
    skipped pairs unchanged)."""
    e = np.asarray(idx, np.int64).reshape(-1)
    lv = np.asarray(level, np.int64).reshape(-1)
    keep = np.ones(e.shape, bool) if skip is None else ~np.asarray(skip, bool).reshape(-1)
    vote = np.full(E, -1, np.int8)
    for x in np.unique(e[keep]):
        sel = lv[keep & (e == x)]
        n = sel.size
        v = 2
        for L in (0, 1):
            if int((sel <= L).sum()) >= (float(hi_vote) - 1e-9) * n:
                v = L
                break
        vote[x] = v
    out = lv.copy()
    out[keep] = vote[e[keep]]
    return vote, out.reshape(np.asarray(level).shape).astype(np.uint8)


def level_to_slot(level: int, n_prec: int) -> int:
    """Level -> index into the store's precision list, most precise first (moelab/policy.py:188-192)."""
    if n_prec >= 3:
        return min(level, n_prec - 1)
    return 0 if level == 0 else n_prec - 1


# ---------------------------------------------------------------------------------------------
# Dispatch (moelab/runtime.py:459-492, `_decide_general`)
# ---------------------------------------------------------------------------------------------

def dispatch(idx: np.ndarray, slot: np.ndarray | None, skip: np.ndarray | None, E: int, P: int = 1):
    """Per-expert and per-(expert, precision slot) pair lists.

    Pairs (t, j) not skipped are flattened to position p = t*k + j. `by_expert` is the stable
    argsort of the kept pairs by expert (the reference's flat_pos[order]), with per-expert counts
    over all E experts (zeros included). `by_key` is the stable sort by key = expert*P + slot.
    Returns dict(counts_e [E], pos_e [n], counts_k [E*P], pos_k [n]).
    """
    T, k = idx.shape
    n = T * k
    keep = np.ones(n, bool) if skip is None else ~np.asarray(skip, bool).reshape(-1)
    e = np.asarray(idx, np.int64).reshape(-1)
    sl = np.zeros(n, np.int64) if slot is None else np.asarray(slot, np.int64).reshape(-1)
    pos = np.arange(n, dtype=np.int64)[keep]
    ek = e[keep]
    key = ek * P + sl[keep]
    oe = np.argsort(ek, kind="stable")
    ok = np.argsort(key, kind="stable")
    return {
        "counts_e": np.bincount(ek, minlength=E).astype(np.int32),
        "pos_e": pos[oe].astype(np.int32),
        "counts_k": np.bincount(key, minlength=E * P).astype(np.int32),
        "pos_k": pos[ok].astype(np.int32),
    }


# ---------------------------------------------------------------------------------------------
# Expert products and combine (moelab/runtime.py:165-168, 335-355, 681-702)
# ---------------------------------------------------------------------------------------------

def silu(a: np.ndarray) -> np.ndarray:
    a = a.astype(np.float32)
    return (a / (np.float32(1) + np.exp(-a))).astype(np.float32)


def expert_ffn_f32(x: np.ndarray, gate_up: np.ndarray, down: np.ndarray) -> np.ndarray:
    """down(silu(gate x) * up x) in float32 (moelab/runtime.py:165-168)."""
    g_u = x.astype(np.float32) @ gate_up.T.astype(np.float32)
    I = gate_up.shape[0] // 2
    return (silu(g_u[:, :I]) * g_u[:, I:]) @ down.T.astype(np.float32)


def shared_expert(x: np.ndarray, wg: np.ndarray, record: np.ndarray, layout: dict, dtype: str) -> np.ndarray:
    """Qwen3-Next shared-expert branch in float32: sigmoid(x . wg) * down(silu(gate x) * up x)
    (transformers qwen3_next/modeling_qwen3_next.py:789-801). The gate logit is rounded to the
    model dtype as F.linear returns it; the shared MLP is one record (gate_up = [gate_proj; up_proj])."""
    xf = np.asarray(x, np.float32)
    g = _round_f64_to(xf.astype(np.float64) @ np.asarray(wg, np.float64), dtype)
    s = (np.float32(1) / (np.float32(1) + np.exp(-g.astype(np.float32)))).astype(np.float32)
    gu, dn = materialize_f32(layout, record)
    return s[:, None] * expert_ffn_f32(xf, gu, dn)


def grouped_ffn(x_row: np.ndarray, records: list, layout: dict, weights: list) -> np.ndarray:
    """sum_e w_e * expert_e(x) for one token, fp32 (the reference kernels' contract,
    moelab/kernels.py:834-872; reference test helper tests/test_kernels.py:23-29)."""
    x = np.asarray(x_row, np.float32).reshape(1, -1)
    out = np.zeros_like(x)
    for b, w in zip(records, weights):
        gu, dn = materialize_f32(layout, b)
        out += np.float32(w) * expert_ffn_f32(x, gu, dn)
    return out


def moe_layer(x: np.ndarray, idx: np.ndarray, w: np.ndarray, slot: np.ndarray | None, skip: np.ndarray | None,
              records: dict, layouts: dict, E: int, cache: dict | None = None) -> np.ndarray:
    """The MoE layer output in float32: out[t] = sum over kept pairs (t, j) of
    w[t,j] * expert_{idx[t,j]}(x[t]) evaluated at the pair's own precision slot.

    records[slot][e] is the uint8 record of expert e at precision slot `slot`, layouts[slot] its
    layout. Follows the CPU expert path (moelab/runtime.py:681-702: materialize to float32,
    expert_ffn, index_add of weighted outputs), with the precision taken per pair instead of
    voted per expert. `cache` memoises dequantised experts across calls.
    """
    T, k = idx.shape
    P = len(layouts)
    d = dispatch(idx, slot, skip, E, P)
    out = np.zeros((T, x.shape[1]), np.float32)
    xf = np.asarray(x, np.float32)
    wf = np.asarray(w, np.float32).reshape(-1)
    start = 0
    for key, c in enumerate(d["counts_k"]):
        if c == 0:
            continue
        pos = d["pos_k"][start:start + c]
        start += c
        e, s = divmod(key, P)
        ck = (s, e)
        if cache is not None and ck in cache:
            gu, dn = cache[ck]
        else:
            gu, dn = materialize_f32(layouts[s], records[s][e])
            if cache is not None:
                cache[ck] = (gu, dn)
        tok = pos // k
        y = expert_ffn_f32(xf[tok], gu, dn)
        np.add.at(out, tok, y * wf[pos][:, None])
    return out


# ---------------------------------------------------------------------------------------------
# Dense int8 layers (moelab/denseq.py)
# ---------------------------------------------------------------------------------------------

def dense_int8_dequant(q: np.ndarray, scales: np.ndarray, dtype: str) -> np.ndarray:
    """moelab's dequantize(q, s, 8, dtype) (quant.py:191-205) as float32 values: q and the fp16
    scale are each converted to `dtype` (q exactly), and their product is rounded once to `dtype`."""
    out_f, in_f = q.shape
    gs = in_f // scales.shape[1]
    qv = round_to(q.astype(np.float32), dtype)
    sv = round_to(scales.astype(np.float32), dtype)
    prod = qv.reshape(out_f, in_f // gs, gs) * sv[..., None]  # exact in fp32 (8-bit x 11-bit)
    return round_to(prod.reshape(out_f, in_f), dtype)


def dense_int8_linear(x: np.ndarray, q: np.ndarray, scales: np.ndarray, bias: np.ndarray | None,
                      dtype: str) -> np.ndarray:
    """QLinear.forward for one decode batch (denseq.py:89-102 with the GEMV `_gemv8`, 34-57): the
    float32 dot products of the int8 weights times their group scales with x, rounded to the
    activation dtype, then + bias in that dtype. Computed in float64 here (the kernel sums in fp32
    in its own order; parity is a tolerance)."""
    w = dequantize(q.view(np.int8) if q.dtype != np.int8 else q, scales, 8).astype(np.float64)
    y = round_to((x.astype(np.float64) @ w.T).astype(np.float32), dtype)
    if bias is not None:
        y = round_to(y + round_to(bias, dtype), dtype)
    return y


def max_rel_err(got: np.ndarray, ref: np.ndarray) -> float:
    """max |got - ref| / max |ref| -- the metric of the reference's kernel tests
    (tests/test_kernels.py:49)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    den = float(np.abs(ref).max())
    return float(np.abs(got - ref).max()) / (den if den > 0 else 1.0)
