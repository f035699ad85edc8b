"""Store-to-device path: cold records read from an expert store on disk into pinned pool slots
(reader threads, while the resident pairs compute), copied to device slots on the copy stream, the
pool slots quarantined until their copy's event and a layer advance (moelab store.py:423-445,
hostpool.py:140-170, runtime.py:310-333). Layer outputs against the all-resident layer and the
oracle; the reference-built tiny store is read end to end."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from gpu_util import TOL, act_np, layer_records
from moeb200 import B200Runtime, ops
from moeb200 import format as F
from moeb200.cold import ColdExperts
from moeb200.hostpool import PinnedPool
from moeb200.store import RecordStore, write_store
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

GOLD = Path(__file__).resolve().parent / "golden" / "store_tiny"


@pytest.mark.parametrize("cap_slots", [64, 3])
def test_stored_cold_layers_match_resident(cuda_dev, tmp_path, cap_slots):
    # two layers in a store written from GPU-quantised records; 40 % of each layer's experts stay
    # on disk; cap_slots = 3 pool slots per precision forces the quarantine to hand slots back
    # between layers (and the pool to lend ordinary buffers when all are held)
    H, I, E, k, T, L = 512, 256, 12, 4, 16, 2
    precs = ["fp16", "int4"]
    recs = [layer_records(precs, H, I, E, seed=60 + li, device=cuda_dev, std=0.05)[1] for li in range(L)]
    lays = {p: F.record_layout(p, H, I) for p in precs}
    path = write_store(tmp_path / "store", [f"layer{li}" for li in range(L)], E, H, I, precs,
                       lambda li, e, p: recs[li][p][e])
    store = RecordStore(path, read_parts=2)
    rb = {p: store.record_bytes(p) for p in precs}
    pool = PinnedPool(rb, cap_bytes=cap_slots * max(rb.values()), slab_bytes=max(rb.values()))
    pol = ops.PolicySpec("threshold", thr=0.3)
    hot = B200Runtime(precs, lays, E, cuda_dev, pol, layers=range(L))
    rt = B200Runtime(precs, lays, E, cuda_dev, pol, layers=range(L))
    cold_set = [e for e in range(E) if e % 5 in (1, 3)]
    for li in range(L):
        for p in precs:
            for e in range(E):
                hot.add_record(li, e, p, recs[li][p][e])
                rt.add_record(li, e, p, recs[li][p][e])
    cold = ColdExperts(rt, {p: len(cold_set) for p in precs}, store=store, pool=pool)
    for li in range(L):
        for e in cold_set:
            for p in precs:
                cold.add_stored(li, e, p)
    g = torch.Generator(device=cuda_dev).manual_seed(13)
    for step in range(3):
        cold.reset()  # every step reads the routed cold records from disk again
        x = torch.randn(T, H, generator=g, device=cuda_dev).half()
        for li in range(L):
            wv, idx = torch.topk(torch.randn(T, E, generator=g, device=cuda_dev).softmax(-1), k, dim=-1)
            lvl, skip = hot.levels(li, wv)
            out = torch.empty_like(x)
            cold.run_layer(li, x, idx, wv, lvl, skip, out)
            ref_dev = hot.run_layer(li, x, idx, wv, level=lvl, skip=skip)
            torch.cuda.synchronize()
            slot = np.vectorize(lambda v: O.level_to_slot(int(v), 2))(lvl.cpu().numpy().astype(np.int64))
            recs_np = [[b.cpu().numpy() for b in recs[li][p]] for p in precs]
            ref = O.moe_layer(act_np(x), idx.cpu().numpy(), wv.cpu().numpy(), slot,
                              skip.cpu().numpy().astype(bool), recs_np, [lays[p] for p in precs], E)
            assert O.max_rel_err(act_np(out), ref) < TOL, (step, li)
            assert O.max_rel_err(act_np(out), act_np(ref_dev)) < 4e-3, (step, li)
            x = (x.float() + out.float()).half()
    assert int(rt.miss.item()) == 0
    assert store.reads > 0 and cold.uploads == store.reads
    if cap_slots == 64:
        assert pool.fallbacks == 0
    store.close()


def test_reference_built_store_end_to_end(cuda_dev):
    # every expert of the reference-built tiny store stays on disk: the layer reads all it needs
    store = RecordStore(GOLD)
    E, H, I = store.num_experts, store.hidden, store.inter
    precs = store.precisions
    lays = {p: store.layouts[p] for p in precs}
    pool = PinnedPool({p: store.record_bytes(p) for p in precs}, cap_bytes=1 << 22)
    rt = B200Runtime(precs, lays, E, cuda_dev, ops.PolicySpec("threshold", thr=0.4), layers=range(len(store.layers)))
    cold = ColdExperts(rt, {p: E for p in precs}, store=store, pool=pool)
    for li in range(len(store.layers)):
        for e in range(E):
            for p in precs:
                cold.add_stored(li, e, p)
    g = torch.Generator(device=cuda_dev).manual_seed(2)
    T, k = 6, 2
    for li in range(len(store.layers)):
        x = torch.randn(T, H, generator=g, device=cuda_dev).half()
        wv, idx = torch.topk(torch.randn(T, E, generator=g, device=cuda_dev).softmax(-1), k, dim=-1)
        lvl, skip = rt.levels(li, wv)
        out = torch.empty_like(x)
        cold.run_layer(li, x, idx, wv, lvl, skip, out)
        torch.cuda.synchronize()
        slot = np.vectorize(lambda v: O.level_to_slot(int(v), 2))(lvl.cpu().numpy().astype(np.int64))
        recs_np = [[store.read(li, e, p).numpy() for e in range(E)] for p in precs]
        ref = O.moe_layer(act_np(x), idx.cpu().numpy(), wv.cpu().numpy(), slot, skip.cpu().numpy().astype(bool),
                          recs_np, [lays[p] for p in precs], E)
        assert O.max_rel_err(act_np(out), ref) < TOL, li
    assert int(rt.miss.item()) == 0 and cold.uploads > 0
    store.close()
