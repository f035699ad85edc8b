"""Cold experts: records held in pinned host memory and uploaded to device slots when routed.

Mirrors moelab's VRAM-miss path for resident-or-host experts: `_to_fast` copies a pinned record
to the device on a dedicated copy stream and records an event, `_ready` makes the compute stream
wait on it before use (moelab/runtime.py:310-333), and the host pool lends pinned slots and only
reuses a slot after the event of its last use (moelab/hostpool.py:52-196).

A cold record is held either in pinned host memory (`add_cold`) or only on disk in an expert store
(`add_stored`, with a moeb200.store.RecordStore and a moeb200.hostpool.PinnedPool): a stored record
that is routed is read by the store's reader threads into a pool slot while the resident pairs
compute, then copied to its device slot on the copy stream; the pool slot goes back with the copy's
event and is reused only after it fired and the pool advanced a layer (moelab's store-to-device
path: ExpertStore.read, store.py:423-445, into HostPool slots, hostpool.py:140-170).

Per layer, `ColdExperts.run_layer` (or `run_part` for the experts [e_lo, e_hi) of one rank of an
expert-parallel group, over the gathered tokens of every rank, writing an fp32 partial sum):
  1. reads the routing back once (the reference reads it back too, moelab/runtime.py:505) and
     lists the (expert, precision) records in range that are routed but only held on the host;
  2. assigns each one a device slot (least recently used first, never a slot that this layer needs)
     and issues one cudaMemcpyAsync per record on the copy stream; a reused slot's copy first waits
     on the event that ended its previous use; one event marks the end of the uploads;
  3. runs the resident (hot) pairs on the compute stream while the copies are in flight, then waits
     on the upload event and runs the uploaded (cold) pairs; both passes write fp32 partial sums
     that are added in a fixed order and cast once (moeb200_combine_parts).
"""

from __future__ import annotations

from collections import OrderedDict

import numpy as np
import torch

from . import ops
from .runtime import aligned_empty


class SlotPlan:
    """Slot bookkeeping of one precision (host logic only, no CUDA): a key is
    (layer, expert, precision); slots are reused least recently used first."""

    def __init__(self, n_slots: int):
        if n_slots <= 0:
            raise ValueError("at least one slot")
        self.n_slots = n_slots
        self.key_of: list[tuple | None] = [None] * n_slots
        self.slot_of: dict[tuple, int] = {}
        self.lru: OrderedDict[int, None] = OrderedDict((i, None) for i in range(n_slots))  # oldest first

    def assign(self, needed: list[tuple]) -> tuple[dict, list]:
        """Slots for every key of `needed` (distinct keys). Returns (slot of each key, uploads) where
        uploads lists (key, slot, evicted key or None) for keys that were not in a slot yet."""
        need = list(dict.fromkeys(needed))
        if len(need) > self.n_slots:
            raise RuntimeError(f"{len(need)} cold records routed at once but only {self.n_slots} device slots")
        res, uploads = {}, []
        for key in need:
            s = self.slot_of.get(key)
            if s is not None:
                res[key] = s
                self.lru.move_to_end(s)
        busy = set(res.values())
        for key in need:
            if key in res:
                continue
            s = next(i for i in self.lru if i not in busy)
            old = self.key_of[s]
            if old is not None:
                del self.slot_of[old]
            self.key_of[s] = key
            self.slot_of[key] = s
            self.lru.move_to_end(s)
            busy.add(s)
            res[key] = s
            uploads.append((key, s, old))
        return res, uploads

    def clear(self) -> list[tuple]:
        """Forget every slot's content; returns the keys that were held."""
        held = [k for k in self.key_of if k is not None]
        self.key_of = [None] * self.n_slots
        self.slot_of.clear()
        return held


class ColdExperts:
    """Host-held records of a B200Runtime, uploaded into `slots[prec]` device slots on demand."""

    def __init__(self, runtime, slots: dict[str, int], store=None, pool=None):
        self.rt = runtime
        self.dev = runtime.device
        self.store = store  # RecordStore of the records added with add_stored
        self.pool = pool    # PinnedPool the stored records are read into
        self.disk: set[tuple] = set()
        self.copy_stream = torch.cuda.Stream(self.dev)
        self.host: dict[tuple, torch.Tensor] = {}
        self.plans = {p: SlotPlan(n) for p, n in slots.items()}
        self.buf = {}
        for p, n in slots.items():
            rb = runtime.layouts[p]["record_bytes"]  # a multiple of 4096: every slot stays aligned
            self.buf[p] = aligned_empty((n, rb), self.dev)
            runtime.note_region(self.buf[p].data_ptr())
        self.last_use: dict[tuple[str, int], torch.cuda.Event] = {}
        self.uploaded_bytes = 0
        self.uploads = 0
        self._codes: dict[int, np.ndarray] = {}

    def add_cold(self, layer: int, expert: int, prec: str, blob: torch.Tensor) -> None:
        """Register a record held on the host (pinned uint8 tensor; pinned here if it is not)."""
        if blob.is_cuda or blob.dtype != torch.uint8:
            raise ValueError("cold records are uint8 host tensors")
        if blob.numel() != self.rt.layouts[prec]["record_bytes"]:
            raise ValueError("record size does not match the precision's layout")
        if prec not in self.plans:
            raise ValueError(f"no device slots for precision {prec}")
        self.host[(layer, expert, prec)] = blob if blob.is_pinned() else blob.pin_memory()
        self._codes.pop(layer, None)
        self.rt.remove_record(layer, expert, prec)

    def add_stored(self, layer: int, expert: int, prec: str) -> None:
        """Register a record that stays on disk in the store (read when routed)."""
        if self.store is None or self.pool is None:
            raise ValueError("stored cold records need a store and a pinned pool")
        if prec not in self.plans:
            raise ValueError(f"no device slots for precision {prec}")
        if self.store.record_bytes(prec) != self.rt.layouts[prec]["record_bytes"]:
            raise ValueError("the store's record size does not match the precision's layout")
        self.disk.add((layer, expert, prec))
        self.host.pop((layer, expert, prec), None)
        self._codes.pop(layer, None)
        self.rt.remove_record(layer, expert, prec)

    def _cold_codes(self, layer: int, E: int, P: int) -> np.ndarray:
        """expert * P + slot of every host-held record of `layer` (cached per layer)."""
        c = self._codes.get(layer)
        if c is None:
            keys = set(self.host) | self.disk
            c = np.array(sorted(e * P + self.rt.precisions.index(p) for (l_, e, p) in keys if l_ == layer), np.int64)
            self._codes[layer] = c
        return c

    def _write_table(self, writes: dict[int, list[tuple[int, int]]]) -> None:
        """Write (flat index p * E + e, record address) entries into each layer's device table with
        one indexed store per layer on the current stream; the index/value pairs go up from pinned
        memory without blocking the host."""
        for layer, ent in writes.items():
            if not ent:
                continue
            iv = torch.tensor(ent, dtype=torch.int64).pin_memory().to(self.dev, non_blocking=True)
            self.rt._table(layer).view(-1).index_put_((iv[:, 0],), iv[:, 1])

    def reset(self) -> None:
        """Drop every uploaded record (their table entries go back to not resident)."""
        E = self.rt.num_experts
        writes: dict[int, list[tuple[int, int]]] = {}
        for p, plan in self.plans.items():
            for (layer, e, prec) in plan.clear():
                writes.setdefault(layer, []).append((self.rt.precisions.index(prec) * E + e, 0))
        self._write_table(writes)

    @torch.no_grad()
    def run_layer(self, layer: int, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, level: torch.Tensor | None,
                  skip: torch.Tensor | None, out: torch.Tensor) -> torch.Tensor:
        """out[T, H] = the layer over every expert, uploading the routed cold records first."""
        return self._run(layer, x, idx, w, level, skip, 0, self.rt.num_experts, out=out)

    @torch.no_grad()
    def run_part(self, layer: int, e_lo: int, e_hi: int, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor,
                 level: torch.Tensor | None, skip: torch.Tensor | None, part: torch.Tensor) -> torch.Tensor:
        """part[T, H] fp32 = the pairs routed to experts [e_lo, e_hi) (one rank's block under expert
        parallelism: the tokens are every rank's), uploading the block's routed cold records first."""
        return self._run(layer, x, idx, w, level, skip, e_lo, e_hi, part=part)

    def _run(self, layer: int, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, level: torch.Tensor | None,
             skip: torch.Tensor | None, e_lo: int, e_hi: int, out: torch.Tensor | None = None,
             part: torch.Tensor | None = None) -> torch.Tensor:
        rt = self.rt
        T, k = idx.shape
        P = rt.n_prec
        # one read-back of the routing (indices, levels, skips)
        rows = [idx.to(torch.int64)]
        if level is not None:
            rows.append(level.to(torch.int64))
        if skip is not None:
            rows.append(skip.to(torch.int64))
        back = torch.stack(rows).cpu().numpy()
        idx_h = back[0]
        lv_h = back[1] if level is not None else np.zeros((T, k), np.int64)
        sk_h = back[-1].astype(bool) if skip is not None else np.zeros((T, k), bool)
        # precision slot of every pair (moelab/policy.py:188-192) and its (expert, slot) code
        slot = np.minimum(lv_h, P - 1) if P >= 3 else np.where(lv_h == 0, 0, P - 1)
        code = idx_h.astype(np.int64) * P + slot
        cold_code = self._cold_codes(layer, rt.num_experts, P)
        cold_pair = np.isin(code, cold_code) & ~sk_h & (idx_h >= e_lo) & (idx_h < e_hi)
        needed: dict[str, list] = {p: [] for p in self.plans}
        for c in np.unique(code[cold_pair]).tolist():
            e, sl = divmod(int(c), P)
            needed[rt.precisions[sl]].append((layer, e, rt.precisions[sl]))
        cold_pair = torch.from_numpy(cold_pair)
        if not cold_pair.any():
            if part is not None:
                rt._table(layer)
                return ops.experts_forward_part(rt._ctables[layer], e_lo, e_hi, x, idx, w, level, skip, part=part,
                                                miss=rt.miss)
            return rt.run_layer(layer, x, idx, w, level=level, skip=skip, out=out)
        E = rt.num_experts
        writes: dict[int, list[tuple[int, int]]] = {}
        cur = torch.cuda.current_stream(self.dev)
        self.copy_stream.wait_stream(cur)  # the routing and any earlier table writes come first
        if self.pool is not None:
            self.pool.advance()  # a new layer: pool slots released by earlier layers may be reused
        used, disk = [], []
        with torch.cuda.stream(self.copy_stream):
            for prec, keys in needed.items():
                if not keys:
                    continue
                slot_of, uploads = self.plans[prec].assign(keys)
                used += [(prec, s) for s in slot_of.values()]
                for key, s, old in uploads:
                    ev = self.last_use.get((prec, s))
                    if key in self.host:
                        if ev is not None:
                            self.copy_stream.wait_event(ev)  # quarantine: the slot's last reader is done
                        self.buf[prec][s].copy_(self.host[key], non_blocking=True)
                        self.uploaded_bytes += self.host[key].numel()
                        self.uploads += 1
                    else:  # on disk: read on a store thread into a pool slot, copied once it is there
                        hb = self.pool.acquire(prec)
                        disk.append((key, prec, s, ev, hb, self.store.read_async(key[0], key[1], prec, hb)))
                    if old is not None:
                        ol, oe, op = old
                        writes.setdefault(ol, []).append((rt.precisions.index(op) * E + oe, 0))
                for (l_, e, p_), s in slot_of.items():
                    writes.setdefault(layer, []).append((rt.precisions.index(p_) * E + e, self.buf[p_][s].data_ptr()))
        mask = cold_pair.to(self.dev, non_blocking=True).to(torch.uint8)
        base = skip if skip is not None else torch.zeros(T, k, dtype=torch.uint8, device=self.dev)
        parts = torch.empty(2, T, x.shape[-1], dtype=torch.float32, device=self.dev)
        ct = rt._ctables[layer]
        # hot pairs run while the uploads (and the disk reads) are in flight: the cold pairs' table
        # entries are written on the copy stream and only read after the compute stream has waited on
        # `done`; the hot pass reads no entry of a cold key
        ops.experts_forward_part(ct, e_lo, e_hi, x, idx, w, level, base | mask, part=parts[0], miss=rt.miss)
        with torch.cuda.stream(self.copy_stream):
            for key, prec, s, ev, hb, fut in disk:
                fut.result()  # the record is in the pool slot
                if ev is not None:
                    self.copy_stream.wait_event(ev)
                self.buf[prec][s].copy_(hb, non_blocking=True)
                copied = torch.cuda.Event()
                copied.record(self.copy_stream)
                self.pool.release(hb, copied)  # reusable after this copy and a layer advance
                self.uploaded_bytes += hb.numel()
                self.uploads += 1
            # one indexed store per table; its entries are distinct (an evicted key is never one that
            # this layer needs, and each slot holds one key)
            self._write_table(writes)
            done = torch.cuda.Event()
            done.record(self.copy_stream)
        cur.wait_event(done)
        ops.experts_forward_part(ct, e_lo, e_hi, x, idx, w, level, base | (1 - mask), part=parts[1], miss=rt.miss)
        for prec, s in used:
            ev = torch.cuda.Event()
            ev.record(cur)
            self.last_use[(prec, s)] = ev
        if part is not None:
            return ops.combine_parts(parts, part)
        ops.combine_parts(parts, out)
        return out
