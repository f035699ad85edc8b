"""The grouped-expert API of moelab/kernels.py, served by the sm_100a kernels of libmoeb200.

Same names, arguments and semantics as the reference (moelab/kernels.py:70-74, 747-769, 834-891):
``entries`` is ``[(views(record), router weight), ...]`` with every record in one layout, the result
is ADDED into ``out`` (1, H), a weight of 0 is a no-op, accumulation is fp32. ``version`` is
accepted for signature compatibility and ignored (there is one kernel family). Unlike the reference
there is no torch fallback: unsupported shapes raise ``MoeB200Error``.
"""

from __future__ import annotations

import torch

from . import _lib, ops
from .format import WTYPE

_KEYS_INT = ("gate_up.q", "gate_up.s", "down.q", "down.s")
_KEYS_FLOAT = ("gate_up", "gate_up", "down", "down")
_FLOAT_WT = {torch.float16: "fp16", torch.bfloat16: "bf16", torch.float32: "fp32"}


class _Staging:
    """Pinned host ring for the pointer tables, so a table upload never waits for the GPU
    (the reference does the same, moelab/kernels.py:195-224)."""

    def __init__(self, slots: int = 32, nbytes: int = 64 * 1024):
        self.bufs = [torch.empty(nbytes, dtype=torch.uint8, pin_memory=True) for _ in range(slots)]
        self.events: list = [None] * slots
        self.i = 0

    def send(self, host: torch.Tensor, device) -> torch.Tensor:
        n = host.numel()
        if n > self.bufs[0].numel():
            return host.to(device)
        i = self.i
        self.i = (i + 1) % len(self.bufs)
        if self.events[i] is not None:
            self.events[i].synchronize()
        buf = self.bufs[i][:n]
        buf.copy_(host)
        dev = torch.empty(n, dtype=torch.uint8, device=device)
        dev.copy_(buf, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self.events[i] = ev
        return dev


_staging: _Staging | None = None


def _table(entries, keys, device) -> tuple[torch.Tensor, torch.Tensor]:
    global _staging
    n = len(entries)
    host = torch.empty(n * 32 + n * 4, dtype=torch.uint8)
    ptrs = []
    for v, _ in entries:
        for k in keys:
            p = v[k].data_ptr()
            if p % 16:
                raise ValueError(f"record field {k} is not 16-byte aligned")
            ptrs.append(p)
    host[: n * 32].view(torch.int64).copy_(torch.tensor(ptrs, dtype=torch.int64))
    host[n * 32:].view(torch.float32).copy_(torch.tensor([float(w) for _, w in entries], dtype=torch.float32))
    if _staging is None:
        _staging = _Staging()
    dev = _staging.send(host, device)
    return dev[: n * 32].view(torch.int64).view(n, 4), dev[n * 32:].view(torch.float32)


def _layout_int(v: dict, bits: int) -> _lib.Layout:
    two_i, cols = v["gate_up.q"].shape
    H = cols * 2 if bits == 4 else cols
    I = two_i // 2
    L = _lib.Layout()
    L.wtype = _lib.I4 if bits == 4 else _lib.I8
    L.hidden, L.inter = H, I
    L.gs_up = H // v["gate_up.s"].shape[1]
    L.gs_dn = I // v["down.s"].shape[1]
    L.off_gu_q = L.off_gu_s = L.off_dn_q = L.off_dn_s = 0  # the table holds field addresses
    return L


def _layout_float(v: dict) -> _lib.Layout:
    two_i, H = v["gate_up"].shape
    L = _lib.Layout()
    L.wtype = WTYPE[_FLOAT_WT[v["gate_up"].dtype]]
    L.hidden, L.inter = H, two_i // 2
    L.off_gu_q = L.off_dn_q = 0
    L.off_gu_s = L.off_dn_s = -1
    return L


def _run(layout_c, entries, keys, x_row, out) -> None:
    if not entries:
        return
    tab, w = _table(entries, keys, x_row.device)
    x = x_row.reshape(-1).contiguous()
    o = out.reshape(-1)
    if not o.is_contiguous():
        raise ValueError("out must be contiguous")
    ops.grouped_ffn_table(layout_c, tab, w, x, o)


def grouped_ffn_int4(x_row: torch.Tensor, entries: list, groups: dict, out: torch.Tensor, version: int = 0) -> None:
    """out (1, H) += sum of int4 experts (moelab/kernels.py:834-872)."""
    if entries:
        _run(_layout_int(entries[0][0], 4), entries, _KEYS_INT, x_row, out)


def grouped_ffn_int8(x_row: torch.Tensor, entries: list, layout: dict, out: torch.Tensor) -> None:
    """out (1, H) += sum of int8 experts (moelab/kernels.py:747-769)."""
    if entries:
        _run(_layout_int(entries[0][0], 8), entries, _KEYS_INT, x_row, out)


def grouped_ffn_float(x_row: torch.Tensor, entries: list, out: torch.Tensor) -> None:
    """out (1, H) += sum of float experts (moelab/kernels.py:875-891)."""
    if entries:
        _run(_layout_float(entries[0][0]), entries, _KEYS_FLOAT, x_row, out)


def expert_ffn_int4(x: torch.Tensor, v: dict, groups: dict, act_fn) -> torch.Tensor:
    """down(silu(gate x) * up x) for one int4 expert and one token (moelab/kernels.py:70-74)."""
    from .runtime import require_silu

    require_silu(act_fn)
    out = torch.zeros(1, x.shape[-1], dtype=x.dtype, device=x.device)
    grouped_ffn_int4(x, [(v, 1.0)], groups, out)
    return out.view_as(x)
