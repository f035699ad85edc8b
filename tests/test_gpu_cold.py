"""Cold experts uploaded from pinned host memory on a copy stream: the layer output equals the
all-resident layer and the oracle, across steps that hit, evict and reuse slots."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from gpu_util import TOL, act_np, layer_records
from moeb200 import B200Runtime, ops
from moeb200.cold import ColdExperts
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n_slots", [16, 5])
def test_cold_layer_matches_resident(cuda_dev, n_slots):
    H, I, E, k, T = 512, 256, 16, 4, 24
    precs = ["fp16", "int4"]
    lays, recs = layer_records(precs, H, I, E, seed=41, device=cuda_dev, std=0.05)
    pol = ops.PolicySpec("threshold", thr=0.3)
    hot_rt = B200Runtime(precs, lays, E, cuda_dev, pol, layers=[0])
    cold_rt = B200Runtime(precs, lays, E, cuda_dev, pol, layers=[0])
    for p in precs:
        for e in range(E):
            hot_rt.add_record(0, e, p, recs[p][e])
            cold_rt.add_record(0, e, p, recs[p][e])
    cold = ColdExperts(cold_rt, {"fp16": n_slots, "int4": n_slots})
    cold_set = [e for e in range(E) if e % 5 in (1, 3)]  # 40 % of the experts
    for e in cold_set:
        for p in precs:
            cold.add_cold(0, e, p, recs[p][e].cpu())
    g = torch.Generator(device=cuda_dev).manual_seed(7)
    recs_np = [[b.cpu().numpy() for b in recs[p]] for p in precs]
    for step in range(3):
        x = torch.randn(T, H, generator=g, device=cuda_dev).half()
        # route only among 4 cold experts per step so a small slot count still fits one layer
        pool = torch.tensor([e for e in range(E) if e not in cold_set] + cold_set[step:step + 4], device=cuda_dev)
        logits = torch.full((T, E), -30.0, device=cuda_dev)
        logits[:, pool] = torch.randn(T, pool.numel(), generator=g, device=cuda_dev)
        wv, idx = torch.topk(logits.softmax(-1), k, dim=-1)
        lvl, skip = hot_rt.levels(0, wv)
        out = torch.empty_like(x)
        cold.run_layer(0, x, idx, wv, lvl, skip, out)
        ref_dev = hot_rt.run_layer(0, x, idx, wv, level=lvl, skip=skip)
        torch.cuda.synchronize()
        slot = np.vectorize(lambda v: O.level_to_slot(int(v), 2))(lvl.cpu().numpy().astype(np.int64))
        ref = O.moe_layer(act_np(x), idx.cpu().numpy(), wv.cpu().numpy(), slot, skip.cpu().numpy().astype(bool),
                          recs_np, [lays[p] for p in precs], E)
        assert O.max_rel_err(act_np(out), ref) < TOL
        assert O.max_rel_err(act_np(out), act_np(ref_dev)) < 4e-3
        assert int(cold_rt.miss.item()) == 0
    assert cold.uploads > 0
    cold.reset()
    assert int((cold_rt._table(0)[:, cold_set] != 0).sum()) == 0


@pytest.mark.parametrize("G", [2, 3])
def test_cold_partials_over_expert_blocks(cuda_dev, G):
    # An expert-parallel rank uploads and runs only its own block [e_lo, e_hi) of the experts over
    # every rank's tokens (ColdExperts.run_part). Here the G blocks run one after another on one GPU,
    # each with its own runtime holding only its block (cold records of the block on the host): the
    # partial sums, added in block order, must match the all-resident layer and the oracle.
    from moeb200.ep import partition

    H, I, E, k, T = 512, 256, 12, 4, 20
    precs = ["fp16", "int4"]
    lays, recs = layer_records(precs, H, I, E, seed=43, device=cuda_dev, std=0.05)
    pol = ops.PolicySpec("threshold", thr=0.3)
    hot_rt = B200Runtime(precs, lays, E, cuda_dev, pol, layers=[0])
    for p in precs:
        for e in range(E):
            hot_rt.add_record(0, e, p, recs[p][e])
    cold_set = [e for e in range(E) if e % 5 in (0, 2)]
    blocks = []
    for r in range(G):
        lo, hi = partition(E, G, r)
        rt = B200Runtime(precs, lays, E, cuda_dev, pol, layers=[0])
        for p in precs:
            for e in range(lo, hi):
                rt.add_record(0, e, p, recs[p][e])
        owned = [e for e in cold_set if lo <= e < hi]
        cold = ColdExperts(rt, {p: max(1, len(owned)) for p in precs})
        for e in owned:
            for p in precs:
                cold.add_cold(0, e, p, recs[p][e].cpu())
        blocks.append((lo, hi, rt, cold))
    g = torch.Generator(device=cuda_dev).manual_seed(9)
    recs_np = [[b.cpu().numpy() for b in recs[p]] for p in precs]
    for step in range(2):
        x = torch.randn(T, H, generator=g, device=cuda_dev).half()
        logits = torch.randn(T, E, generator=g, device=cuda_dev)
        wv, idx = torch.topk(logits.softmax(-1), k, dim=-1)
        lvl, skip = hot_rt.levels(0, wv)
        parts = torch.empty(G, T, H, dtype=torch.float32, device=cuda_dev)
        for r, (lo, hi, rt, cold) in enumerate(blocks):
            cold.reset()
            cold.run_part(0, lo, hi, x, idx, wv, lvl, skip, parts[r])
        out = torch.empty_like(x)
        ops.combine_parts(parts, out)
        ref_dev = hot_rt.run_layer(0, x, idx, wv, level=lvl, skip=skip)
        torch.cuda.synchronize()
        slot = np.vectorize(lambda v: O.level_to_slot(int(v), 2))(lvl.cpu().numpy().astype(np.int64))
        ref = O.moe_layer(act_np(x), idx.cpu().numpy(), wv.cpu().numpy(), slot, skip.cpu().numpy().astype(bool),
                          recs_np, [lays[p] for p in precs], E)
        assert O.max_rel_err(act_np(out), ref) < TOL
        assert O.max_rel_err(act_np(out), act_np(ref_dev)) < 4e-3
    assert sum(c.uploads for _, _, _, c in blocks) > 0
    assert all(int(rt.miss.item()) == 0 for _, _, rt, _ in blocks)
