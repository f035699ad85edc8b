"""Pinned host pool: record-sized slots carved out of large pinned slabs, lent to disk reads and
given back with the event of the device copy that reads them.

The reuse rule is moelab's HostPool (moelab/hostpool.py:52-196: acquire 140-155, release 157-165,
advance 167-170): a released slot is quarantined and becomes free again only when the event it was
released with has completed (the host-to-device copy reading it is over) AND the pool has advanced
at least once since (the caller advances at the start of every layer), so no slot is rewritten
while a copy may still read it. The slab policy is this build's own: slabs of `slab_bytes` (or one
record when that is larger), every slot a multiple of 4096 bytes, up to `cap_bytes`; when the cap is
reached a slab whose slots are all free may be re-carved for another precision; when nothing is
left, acquire lends an ordinary (unpinned, 4096-byte aligned) buffer and counts a fallback.
"""

from __future__ import annotations

import threading

import torch

SLAB_BYTES = 256 << 20


def _aligned_host(nbytes: int) -> torch.Tensor:
    raw = torch.empty(nbytes + 4096, dtype=torch.uint8)
    off = (-raw.data_ptr()) % 4096
    return raw[off:off + nbytes]


class PinnedPool:
    def __init__(self, record_bytes: dict[str, int], cap_bytes: int, pin: bool = True, slab_bytes: int = SLAB_BYTES):
        for p, rb in record_bytes.items():
            if rb <= 0 or rb % 4096:
                raise ValueError(f"record bytes of {p} must be a positive multiple of 4096")
        self.record_bytes = dict(record_bytes)
        self.cap = int(cap_bytes)
        self.pin = pin
        self.slab_bytes = int(slab_bytes)
        self.lock = threading.Lock()
        self.slabs: list[dict] = []  # {"mem": tensor, "prec": str, "slots": [tensor]}
        self.allocated = 0
        self.free: dict[str, list[torch.Tensor]] = {p: [] for p in record_bytes}
        self.quarantine: list[tuple[torch.Tensor, str, object, int]] = []  # (slot, prec, event, epoch)
        self.owner: dict[int, str] = {}  # slot address -> precision
        self.lent: set[int] = set()
        self.epoch = 0
        self.fallbacks = 0
        self.recarves = 0

    def _carve(self, slab: dict, prec: str) -> None:
        rb = self.record_bytes[prec]
        mem = slab["mem"]
        slab["prec"] = prec
        slab["slots"] = [mem[j * rb:(j + 1) * rb] for j in range(mem.numel() // rb)]
        for s in slab["slots"]:
            self.owner[s.data_ptr()] = prec
            self.free[prec].append(s)

    def _new_slab(self, prec: str) -> bool:
        rb = self.record_bytes[prec]
        size = max(rb, self.slab_bytes // rb * rb)
        if self.allocated + size > self.cap:
            size = (self.cap - self.allocated) // rb * rb
            if size < rb:
                return False
        try:
            mem = torch.empty(size, dtype=torch.uint8, pin_memory=True) if self.pin else _aligned_host(size)
        except RuntimeError:  # the system refused more pinned memory
            self.cap = self.allocated
            return False
        slab = {"mem": mem, "prec": prec, "slots": []}
        self.slabs.append(slab)
        self.allocated += size
        self._carve(slab, prec)
        return True

    def _recarve(self, prec: str) -> bool:
        rb = self.record_bytes[prec]
        for slab in self.slabs:
            other = slab["prec"]
            if other == prec or slab["mem"].numel() < rb:
                continue
            ptrs = {s.data_ptr() for s in slab["slots"]}
            if not ptrs <= {s.data_ptr() for s in self.free[other]}:
                continue  # a slot of it is lent or quarantined
            self.free[other] = [s for s in self.free[other] if s.data_ptr() not in ptrs]
            for ptr in ptrs:
                self.owner.pop(ptr, None)
            self._carve(slab, prec)
            self.recarves += 1
            return True
        return False

    def _sweep(self) -> None:
        keep = []
        for slot, prec, ev, epoch in self.quarantine:
            if epoch < self.epoch and (ev is None or ev.query()):
                self.free[prec].append(slot)
            else:
                keep.append((slot, prec, ev, epoch))
        self.quarantine = keep

    def acquire(self, prec: str) -> torch.Tensor:
        """A uint8 host buffer of exactly one `prec` record (callable from reader threads)."""
        with self.lock:
            if not self.free[prec]:
                self._sweep()
            if not self.free[prec]:
                self._new_slab(prec)
            if not self.free[prec]:
                self._sweep()
                self._recarve(prec)
            if self.free[prec]:
                slot = self.free[prec].pop()
                self.lent.add(slot.data_ptr())
                return slot
            self.fallbacks += 1
        return _aligned_host(self.record_bytes[prec])

    def release(self, slot: torch.Tensor, event=None) -> None:
        """Give a buffer back; `event` (anything with .query()) marks the end of the copy reading it.
        A buffer that is not a pool slot, or is not lent, is ignored."""
        ptr = slot.data_ptr()
        with self.lock:
            prec = self.owner.get(ptr)
            if prec is None or ptr not in self.lent:
                return
            self.lent.discard(ptr)
            self.quarantine.append((slot, prec, event, self.epoch))

    def advance(self) -> None:
        """Start of a layer: slots released before now may be reused once their events completed."""
        with self.lock:
            self.epoch += 1

    def is_pooled(self, buf: torch.Tensor) -> bool:
        return buf.data_ptr() in self.owner

    def n_free(self, prec: str) -> int:
        with self.lock:
            return len(self.free[prec])

    def close(self) -> None:
        with self.lock:
            self.free = {p: [] for p in self.record_bytes}
            self.quarantine.clear()
            self.owner.clear()
            self.lent.clear()
            self.slabs.clear()
            self.allocated = 0
