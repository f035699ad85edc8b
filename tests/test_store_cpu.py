"""Expert store and pinned pool, host side: the reader against a store written by the reference's
own build_store (tests/golden/store_tiny, made by tests/golden/make_store_golden.py), the writer
against the same files, and the pool's quarantine rule (moelab/hostpool.py:140-170) with fake
events. No GPU: the pool runs with unpinned slabs here."""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from moeb200 import format as F
from moeb200.hostpool import PinnedPool
from moeb200.store import RecordStore, StoreError, write_store

GOLD = Path(__file__).resolve().parent / "golden"
STORE = GOLD / "store_tiny"
META = json.loads((GOLD / "store_tiny_meta.json").read_text())


def test_reads_the_reference_store_byte_exact():
    st = RecordStore(STORE, read_parts=1)
    assert st.num_experts == META["num_experts"] and st.hidden == META["hidden"] and st.inter == META["inter"]
    assert st.precisions == META["precisions"]
    for p in st.precisions:
        assert st.layouts[p] == F.record_layout(p, st.hidden, st.inter, 64, st.layouts[p].get("scale"))
    for key, digest in META["record_sha256"].items():
        li, e, p = key.split(":")
        blob = st.read(int(li), int(e), p)
        assert hashlib.sha256(blob.numpy().tobytes()).hexdigest() == digest, key
        # split reads (4096-byte aligned pieces on the reader threads) give the same bytes
        out = torch.empty(st.record_bytes(p), dtype=torch.uint8)
        assert torch.equal(st.read(int(li), int(e), p, out=out, parts=3), blob)
        fut = st.read_async(int(li), int(e), p, torch.empty_like(blob))
        assert torch.equal(fut.result(), blob)
    assert st.reads > 0 and st.bytes_read > 0
    st.close()


def test_bad_requests_and_stores_are_refused(tmp_path):
    st = RecordStore(STORE)
    with pytest.raises(IndexError):
        st.read(0, st.num_experts, "int4")
    with pytest.raises(KeyError):
        st.read(0, 0, "int8")
    with pytest.raises(ValueError):
        st.read(0, 0, "int4", out=torch.empty(7, dtype=torch.uint8))
    st.close()
    with pytest.raises(StoreError):
        RecordStore(tmp_path)  # no manifest
    man = json.loads((STORE / "manifest.json").read_text())
    man["complete"] = False
    (tmp_path / "manifest.json").write_text(json.dumps(man))
    with pytest.raises(StoreError):
        RecordStore(tmp_path)
    man["complete"] = True
    man["layouts"][1]["record_bytes"] += 4096  # a layout the kernels cannot read
    (tmp_path / "manifest.json").write_text(json.dumps(man))
    with pytest.raises(StoreError):
        RecordStore(tmp_path)


def test_writer_reproduces_the_reference_files(tmp_path):
    ref = RecordStore(STORE)
    out = write_store(tmp_path / "s", ref.layers, ref.num_experts, ref.hidden, ref.inter, ref.precisions,
                      lambda li, e, p: ref.read(li, e, p), model_type="olmoe")
    for li in range(len(ref.layers)):
        for p in ref.precisions:
            assert (out / ref.file(li, p).name).read_bytes() == ref.file(li, p).read_bytes()
    mine = json.loads((out / "manifest.json").read_text())
    theirs = json.loads((STORE / "manifest.json").read_text())
    for k in ("format", "version", "layers", "num_experts", "hidden", "inter", "complete"):
        assert mine[k] == theirs[k], k
    assert [lay["fields"] for lay in mine["layouts"]] == [lay["fields"] for lay in theirs["layouts"]]
    back = RecordStore(out)
    assert torch.equal(back.read(1, 2, "int4"), ref.read(1, 2, "int4"))
    ref.close()
    back.close()


class FakeEvent:
    def __init__(self, done: bool = False):
        self.done = done

    def query(self) -> bool:
        return self.done


def test_pool_quarantine_waits_for_event_and_layer_advance():
    pool = PinnedPool({"int4": 4096, "fp16": 8192}, cap_bytes=4 * 4096, pin=False, slab_bytes=2 * 4096)
    a, b = pool.acquire("int4"), pool.acquire("int4")
    assert a.data_ptr() != b.data_ptr() and pool.is_pooled(a) and a.numel() == 4096
    assert a.data_ptr() % 4096 == 0
    ev = FakeEvent(False)
    pool.release(a, ev)
    pool.release(a, ev)  # a second release of the same slot is ignored
    # not reusable in the same layer, nor before its copy finished
    c = pool.acquire("int4")  # a new slab (cap allows 4 slots)
    assert c.data_ptr() not in (a.data_ptr(), b.data_ptr())
    pool.advance()
    d = pool.acquire("int4")
    assert d.data_ptr() != a.data_ptr()  # event still pending
    ev.done = True
    e = pool.acquire("int4")  # cap reached: the quarantined slot is swept back
    assert e.data_ptr() == a.data_ptr()
    # nothing free and the cap reached: an ordinary aligned buffer, counted
    f = pool.acquire("int4")
    assert not pool.is_pooled(f) and pool.fallbacks == 1 and f.numel() == 4096
    pool.release(f)  # not a pool slot: ignored
    pool.close()


def test_pool_recarves_a_free_slab_for_another_precision():
    pool = PinnedPool({"int4": 4096, "fp16": 8192}, cap_bytes=2 * 4096, pin=False, slab_bytes=2 * 4096)
    a = pool.acquire("int4")
    pool.release(a, None)
    pool.advance()
    assert pool.n_free("int4") == 1  # the other slot; `a` is swept on the next acquire
    h = pool.acquire("fp16")  # cap reached: the all-free int4 slab is re-carved into one fp16 slot
    assert pool.is_pooled(h) and h.numel() == 8192 and pool.recarves == 1
    assert pool.fallbacks == 0
    pool.close()


def test_pool_rejects_unaligned_records():
    with pytest.raises(ValueError):
        PinnedPool({"int4": 1000}, cap_bytes=1 << 20, pin=False)
