"""Expert record format: moelab's packed int4/int8 group-size-64 records, produced and viewed here.

The format is a contract with moelab's store (moelab/store.py:36-174, moelab/quant.py:43-127), so the
field table, the packing and the scale choice follow it step for step:
  - a record is one uint8 blob: gate_up [2I, H] then down [H, I]; int precisions store ``.q`` then
    ``.s`` (one fp16 scale per group of ``gs`` input columns); each field starts on a 64-byte
    boundary and the record is padded to 4096 bytes;
  - int4 packs two values per byte, stored +8 in [0, 15], low nibble = even column;
  - the scale of a group is max|w|/qmax ("absmax") or the best of 32 candidates ("mse", the
    store's default for int4), rounded to fp16 before quantising and never zero.
Integer records are quantised on the GPU by the library's own quantiser kernel (csrc/quant.cu); it
is offline work, not part of the MoE-layer hot path.
"""

from __future__ import annotations

import torch

from . import _lib

ALIGN = 4096
FIELD_ALIGN = 64

PRECISIONS = {
    "fp32": {"kind": "float", "dtype": "float32"},
    "fp16": {"kind": "float", "dtype": "float16"},
    "bf16": {"kind": "float", "dtype": "bfloat16"},
    "int8": {"kind": "int", "bits": 8},
    "int4": {"kind": "int", "bits": 4},
}
TORCH_DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16,
                "int8": torch.int8, "uint8": torch.uint8}
ELEM_SIZE = {"float32": 4, "float16": 2, "bfloat16": 2, "int8": 1, "uint8": 1}
WTYPE = {"fp32": _lib.F32, "fp16": _lib.F16, "bf16": _lib.BF16, "int8": _lib.I8, "int4": _lib.I4}
ACT_TYPE = {torch.float16: _lib.F16, torch.bfloat16: _lib.BF16, torch.float32: _lib.F32}


def _align(n: int, a: int) -> int:
    return (n + a - 1) // a * a


def pick_group_size(in_features: int, preferred: int = 64) -> int:
    """Largest even group size <= preferred dividing in_features (moelab/quant.py:49-54)."""
    for gs in range(min(preferred, in_features), 1, -1):
        if in_features % gs == 0 and gs % 2 == 0:
            return gs
    raise ValueError(f"no even group size divides {in_features}")


def record_layout(prec: str, hidden: int, inter: int, group_size: int = 64, scale: str | None = None) -> dict:
    """Field table of one record, same dict as moelab.store.record_layout (store.py:76-115)."""
    spec = PRECISIONS[prec]
    if spec["kind"] == "int" and scale is None:
        scale = "mse" if spec["bits"] == 4 else "absmax"
    mats = {"gate_up": (2 * inter, hidden), "down": (hidden, inter)}
    raw: list[tuple[str, tuple[int, ...], str]] = []
    groups: dict[str, int] = {}
    if spec["kind"] == "float":
        for name, shape in mats.items():
            raw.append((name, shape, spec["dtype"]))
    else:
        bits = spec["bits"]
        for name, (o, i) in mats.items():
            gs = pick_group_size(i, group_size)
            groups[name] = gs
            raw.append((f"{name}.q", (o, i) if bits == 8 else (o, i // 2), "int8" if bits == 8 else "uint8"))
            raw.append((f"{name}.s", (o, i // gs), "float16"))
    fields, off = [], 0
    for name, shape, dt in raw:
        fields.append([name, list(shape), dt, off])
        nbytes = ELEM_SIZE[dt]
        for s in shape:
            nbytes *= s
        off = _align(off + nbytes, FIELD_ALIGN)
    lay = {"precision": prec, "fields": fields, "record_bytes": _align(off, ALIGN), "group_sizes": groups}
    if spec["kind"] == "int":
        lay["scale"] = scale
    return lay


def layout_dims(layout: dict) -> tuple[int, int]:
    """(hidden, inter) of a layout."""
    f = {n: s for n, s, _, _ in layout["fields"]}
    if "down" in f:
        hidden, inter = f["down"]
    else:
        hidden = f["down.q"][0]
        inter = f["gate_up.q"][0] // 2
    return hidden, inter


def to_c(layout: dict) -> _lib.Layout:
    """moelab layout dict -> moeb200_layout."""
    hidden, inter = layout_dims(layout)
    offs = {n: o for n, _, _, o in layout["fields"]}
    L = _lib.Layout()
    L.wtype = WTYPE[layout["precision"]]
    L.hidden, L.inter = hidden, inter
    g = layout.get("group_sizes") or {}
    L.gs_up, L.gs_dn = g.get("gate_up", 0), g.get("down", 0)
    if "gate_up" in offs:
        L.off_gu_q, L.off_gu_s, L.off_dn_q, L.off_dn_s = offs["gate_up"], -1, offs["down"], -1
    else:
        L.off_gu_q, L.off_gu_s = offs["gate_up.q"], offs["gate_up.s"]
        L.off_dn_q, L.off_dn_s = offs["down.q"], offs["down.s"]
    L.record_bytes = layout["record_bytes"]
    return L


def field_offsets(layout: dict) -> list[int]:
    """[gate_up.q, gate_up.s, down.q, down.s] offsets (float records: [gate_up, gate_up, down, down]),
    the pointer-table order of moelab/kernels.py:230-244."""
    offs = {n: o for n, _, _, o in layout["fields"]}
    if "gate_up" in offs:
        return [offs["gate_up"], offs["gate_up"], offs["down"], offs["down"]]
    return [offs["gate_up.q"], offs["gate_up.s"], offs["down.q"], offs["down.s"]]


def views(layout: dict, blob: torch.Tensor) -> dict[str, torch.Tensor]:
    """Typed zero-copy views into a record (moelab/store.py:153-161)."""
    out = {}
    for name, shape, dt, off in layout["fields"]:
        nbytes = ELEM_SIZE[dt]
        for s in shape:
            nbytes *= s
        part = blob[off:off + nbytes]
        if dt != "uint8":
            part = part.view(TORCH_DTYPES[dt])
        out[name] = part.view(shape)
    return out


def encode_record(layout: dict, gate_up: torch.Tensor, down: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Record bytes from float weights (moelab/store.py:122-150), on the weights' device.

    Integer precisions are quantised by the B200 quantiser (``moeb200_quantize``: moelab's absmax /
    mse scale search, byte-identical integers and scales), so they need CUDA tensors; float
    precisions are a plain cast into the record's fields. ``out`` (uint8, record_bytes) is filled in
    place when given."""
    spec = PRECISIONS[layout["precision"]]
    dev = gate_up.device
    if spec["kind"] == "int" and dev.type != "cuda":
        raise ValueError("integer records are quantised on the GPU: pass CUDA tensors")
    buf = out if out is not None else torch.empty(layout["record_bytes"], dtype=torch.uint8, device=dev)
    buf.zero_()
    v = views(layout, buf)
    if spec["kind"] == "float":
        dt = TORCH_DTYPES[spec["dtype"]]
        v["gate_up"].copy_(gate_up.to(dt))
        v["down"].copy_(down.to(dt))
        return buf
    from . import ops

    method = layout.get("scale") or "absmax"
    method = "absmax" if method == "gptq" else method
    for name, w in (("gate_up", gate_up), ("down", down)):
        q, s = ops.quantize(w.contiguous(), spec["bits"], layout["group_sizes"][name], method)
        v[f"{name}.q"].copy_(q.view(v[f"{name}.q"].dtype))
        v[f"{name}.s"].copy_(s)
    return buf
