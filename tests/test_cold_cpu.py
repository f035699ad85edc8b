"""Slot bookkeeping of the cold-expert uploads (host logic, no GPU): hits keep their slot, misses
take the least recently used slot that the current layer does not need, evictions are reported,
and a layer needing more records than slots is refused."""

from __future__ import annotations

import pytest

from moeb200.cold import SlotPlan


def test_hits_and_lru_eviction():
    plan = SlotPlan(3)
    a, b, c, d = [(0, e, "int4") for e in range(4)]
    res, up = plan.assign([a, b])
    assert set(res) == {a, b} and [u[0] for u in up] == [a, b] and all(u[2] is None for u in up)
    res2, up2 = plan.assign([a, c])  # a hits, c takes the free slot
    assert res2[a] == res[a] and [u[0] for u in up2] == [c]
    res3, up3 = plan.assign([d])  # LRU is b (a and c were used more recently)
    assert up3 == [(d, res[b], b)]
    res4, up4 = plan.assign([a, d, b])  # b evicts the LRU slot not needed now: c's
    assert up4 == [(b, res2[c], c)]
    assert len(set(res4.values())) == 3


def test_duplicates_and_capacity():
    plan = SlotPlan(2)
    k = [(1, 5, "fp16"), (1, 5, "fp16"), (1, 6, "fp16")]
    res, up = plan.assign(k)
    assert len(res) == 2 and len(up) == 2
    with pytest.raises(RuntimeError):
        plan.assign([(1, e, "fp16") for e in range(3)])
    held = plan.clear()
    assert sorted(held) == [(1, 5, "fp16"), (1, 6, "fp16")]
    _, up = plan.assign([(1, 5, "fp16")])
    assert up[0][2] is None
