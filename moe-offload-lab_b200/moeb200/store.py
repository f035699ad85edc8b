"""On-disk expert store in moelab's format, read straight into (pinned) host buffers.

The store is a directory (the format of moelab/store.py:1-17, written by its build_store 466-560 and
read by ExpertStore 264-445):

  manifest.json              {"format": "moelab-expert-store", "version": 1, "store_id", "layers":
                              [module prefixes], "num_experts", "hidden", "inter", "layouts":
                              [record layouts, most precise first], "complete": true, ...}
  layer{L:03d}.{prec}.bin    the layer's E records of one precision; record e at byte e * record_bytes

A record is the same uint8 blob the kernels read from device memory (moeb200.format), so reading an
expert is one contiguous read of record_bytes (a multiple of 4096) at a 4096-byte aligned offset.
`RecordStore.read` fills a caller's buffer, optionally in `parts` concurrent 4096-byte aligned
pieces (an SSD gives its bandwidth only with several reads in flight); `read_async` does the same on
the store's reader threads (os.preadv releases the interpreter lock) and returns a future, so the
caller can keep the GPU busy while the disk works. `write_store` writes the same format.
"""

from __future__ import annotations

import hashlib
import json
import os
import threading
import time
from concurrent.futures import Future, ThreadPoolExecutor
from pathlib import Path
from typing import Callable

import numpy as np
import torch

from . import format as F

FORMAT = "moelab-expert-store"
VERSION = 1
ALIGN = F.ALIGN


def _layout_key(lay: dict) -> tuple:
    """What must agree between a stored layout and the kernels' layout: precision, field table,
    record size and group sizes (the scale method is provenance only)."""
    return (lay["precision"], [list(map(lambda v: list(v) if isinstance(v, (list, tuple)) else v, f))
                               for f in lay["fields"]], lay["record_bytes"], dict(lay.get("group_sizes") or {}))


class StoreError(RuntimeError):
    """A store that is missing, incomplete, of another format, or whose layouts the kernels cannot read."""


class RecordStore:
    """Read access to a store directory. Thread-safe: every thread has its own file descriptors."""

    def __init__(self, path: str | Path, read_parts: int = 1, threads: int = 8):
        self.path = Path(path)
        mpath = self.path / "manifest.json"
        if not mpath.exists():
            raise StoreError(f"no manifest.json in {self.path}")
        man = json.loads(mpath.read_text(encoding="utf-8"))
        if man.get("format") != FORMAT or man.get("version") != VERSION:
            raise StoreError(f"{self.path}: not a {FORMAT} v{VERSION} store")
        if not man.get("complete"):
            raise StoreError(f"{self.path}: the store is incomplete")
        self.manifest = man
        self.layers: list[str] = list(man["layers"])
        self.num_experts: int = int(man["num_experts"])
        self.hidden: int = int(man["hidden"])
        self.inter: int = int(man["inter"])
        self.precisions: list[str] = [lay["precision"] for lay in man["layouts"]]
        self.layouts: dict[str, dict] = {}
        for lay in man["layouts"]:
            gs = (lay.get("group_sizes") or {}).get("gate_up", 64)
            ours = F.record_layout(lay["precision"], self.hidden, self.inter, gs, lay.get("scale"))
            if _layout_key(ours) != _layout_key(lay):
                raise StoreError(f"{self.path}: the {lay['precision']} layout differs from the kernels' record layout")
            self.layouts[lay["precision"]] = ours
        self.read_parts = max(1, int(read_parts))
        self._local = threading.local()
        self._fds: list[int] = []
        self._lock = threading.Lock()
        self._pool = ThreadPoolExecutor(max_workers=max(1, threads), thread_name_prefix="moeb200-store")
        self.bytes_read = 0
        self.read_seconds = 0.0
        self.reads = 0

    @property
    def store_id(self) -> str:
        return self.manifest.get("store_id", "")

    def record_bytes(self, prec: str) -> int:
        return self.layouts[prec]["record_bytes"]

    def file(self, layer: int, prec: str) -> Path:
        return self.path / f"layer{layer:03d}.{prec}.bin"

    def _fd(self, path: Path) -> int:
        fds = getattr(self._local, "fds", None)
        if fds is None:
            fds = self._local.fds = {}
        fd = fds.get(path)
        if fd is None:
            fd = fds[path] = os.open(path, os.O_RDONLY)
            with self._lock:
                self._fds.append(fd)
        return fd

    def _read_range(self, path: Path, offset: int, out: torch.Tensor) -> None:
        view = memoryview(out.numpy()).cast("B")
        fd = self._fd(path)
        done = 0
        while done < len(view):
            got = os.preadv(fd, [view[done:]], offset + done)
            if got <= 0:
                raise StoreError(f"short read: {path} at {offset + done} ({done}/{len(view)} bytes)")
            done += got

    def _check(self, layer: int, expert: int, prec: str, out: torch.Tensor | None) -> tuple[int, torch.Tensor]:
        if prec not in self.layouts:
            raise KeyError(f"precision {prec} is not in the store (has {self.precisions})")
        if not 0 <= layer < len(self.layers) or not 0 <= expert < self.num_experts:
            raise IndexError(f"(layer {layer}, expert {expert}) outside the store")
        rb = self.record_bytes(prec)
        if out is None:
            out = torch.empty(rb, dtype=torch.uint8)
        if out.dtype != torch.uint8 or out.is_cuda or out.numel() != rb or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous uint8 host tensor of {rb} bytes")
        return rb, out

    def read(self, layer: int, expert: int, prec: str, out: torch.Tensor | None = None,
             parts: int | None = None) -> torch.Tensor:
        """Record (layer, expert, prec) read into `out` (a uint8 host tensor of record_bytes, e.g. a
        pinned pool slot; allocated when None), in `parts` concurrent aligned pieces."""
        rb, out = self._check(layer, expert, prec, out)
        path, offset = self.file(layer, prec), expert * rb
        parts = self.read_parts if parts is None else max(1, int(parts))
        t0 = time.perf_counter()
        if parts > 1 and rb >= 2 * ALIGN:
            per = -(-rb // parts)  # ceil(rb / parts), then up to whole 4096-byte blocks
            chunk = -(-per // ALIGN) * ALIGN
            futs = [self._pool.submit(self._read_range, path, offset + o, out[o:min(o + chunk, rb)])
                    for o in range(0, rb, chunk)]
            for f in futs:
                f.result()
        else:
            self._read_range(path, offset, out)
        dt = time.perf_counter() - t0
        with self._lock:
            self.bytes_read += rb
            self.read_seconds += dt
            self.reads += 1
        return out

    def read_async(self, layer: int, expert: int, prec: str, out: torch.Tensor) -> Future:
        """read() on one of the store's threads; the future's result is `out`."""
        self._check(layer, expert, prec, out)
        return self._pool.submit(self.read, layer, expert, prec, out, 1)

    def close(self) -> None:
        self._pool.shutdown(wait=True)
        with self._lock:
            for fd in self._fds:
                os.close(fd)
            self._fds.clear()
        self._local = threading.local()


def write_store(path: str | Path, layers: list[str], num_experts: int, hidden: int, inter: int,
                precisions: list[str], record: Callable[[int, int, str], np.ndarray | torch.Tensor],
                model_type: str = "moe", group_size: int = 64) -> Path:
    """Write a store of `record(layer_index, expert, prec)` blobs (uint8, record_bytes each) in the
    format above; precisions are ordered most precise first, as the reader expects."""
    order = ["fp32", "fp16", "bf16", "int8", "int4"]
    precisions = sorted(dict.fromkeys(precisions), key=order.index)
    out = Path(path)
    out.mkdir(parents=True, exist_ok=True)
    lays = [F.record_layout(p, hidden, inter, group_size) for p in precisions]
    ident = json.dumps([model_type, list(layers), num_experts, hidden, inter,
                        [[lay["precision"], lay["record_bytes"]] for lay in lays]])
    man = {"format": FORMAT, "version": VERSION, "store_id": hashlib.sha1(ident.encode()).hexdigest()[:12],
           "model_type": model_type, "layers": list(layers), "num_experts": num_experts, "hidden": hidden,
           "inter": inter, "layouts": lays, "complete": False}
    (out / "manifest.json").write_text(json.dumps(man, indent=1), encoding="utf-8")
    for li in range(len(layers)):
        for lay in lays:
            rb = lay["record_bytes"]
            with open(out / f"layer{li:03d}.{lay['precision']}.bin", "wb") as f:
                for e in range(num_experts):
                    blob = record(li, e, lay["precision"])
                    arr = blob.detach().cpu().numpy() if isinstance(blob, torch.Tensor) else np.asarray(blob)
                    if arr.dtype != np.uint8 or arr.size != rb:
                        raise ValueError(f"record ({li}, {e}, {lay['precision']}) is not {rb} uint8 bytes")
                    f.write(arr.tobytes())
    man["complete"] = True
    (out / "manifest.json").write_text(json.dumps(man, indent=1), encoding="utf-8")
    return out
