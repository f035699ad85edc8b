"""Expert-parallel data flow on CPU gloo ranks (world size 2 and 3): the partition, the dispatch
all_gather of exchange rows, the combine all_to_all and the rank-order sum give, on every rank,
the single-process layer output for that rank's tokens."""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]

H, I, E, K, T = 128, 64, 8, 3, 5


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model(seed: int = 0):
    from oracle import moe_oracle as O

    rng = np.random.default_rng(seed)
    lays = [O.record_layout("fp16", H, I), O.record_layout("int4", H, I)]
    recs = [[], []]
    for _ in range(E):
        gu = (rng.standard_normal((2 * I, H)) * 0.05).astype(np.float32)
        dn = (rng.standard_normal((H, I)) * 0.05).astype(np.float32)
        for s, lay in enumerate(lays):
            recs[s].append(O.encode_record(lay, gu, dn))
    wr = (rng.standard_normal((E, H)) * 0.05).astype(np.float32)
    return lays, recs, wr


def _tokens(rank: int, wr):
    from oracle import moe_oracle as O

    rng = np.random.default_rng(100 + rank)
    x = rng.standard_normal((T, H)).astype(np.float16).astype(np.float32)
    _, w, idx, _ = O.router(x, wr, K, False, "float16")
    level, skip = O.threshold_levels(w, 0.3)
    skip = skip.copy()
    skip[0, K - 1] = True  # one dropped pair
    return x, idx.astype(np.int64), w.astype(np.float32), level.astype(np.uint8), skip.astype(np.uint8)


def _worker(rank: int, world: int, port: int, q, vote: bool = False):
    sys.path[:0] = [str(ROOT), str(ROOT / "moe-offload-lab_b200")]
    import torch.distributed as dist

    from moeb200 import ep
    from oracle import moe_oracle as O
    from tests import ep_util

    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        lays, recs, wr = _model()
        lo, hi = ep.partition(E, world, rank)
        own = [[r if lo <= e < hi else None for e, r in enumerate(rs)] for rs in recs]
        rt = ep_util.CpuRuntime(E, lays, own, 2)
        if vote:  # the per-expert vote, taken over every rank's tokens after the gather
            from types import SimpleNamespace

            rt.policy = SimpleNamespace(hi_vote=0.5)
            rt.votes = lambda layer: True
        par = ep.ExpertParallel(rt, ops=ep_util.CpuOps())
        x, idx, w, level, skip = _tokens(rank, wr)
        if vote:  # three per-pair levels to vote on
            level = O.hobbit_levels(w, t1=0.4, t_mid=0.7)[0].astype(np.uint8)
        xt = torch.from_numpy(x).half()
        out = par.run_layer(0, xt, torch.from_numpy(idx), torch.from_numpy(w), torch.from_numpy(level),
                            torch.from_numpy(skip))
        if vote:
            allt = [_tokens(r, wr) for r in range(world)]
            all_idx = np.concatenate([a[1] for a in allt])
            all_lvl = np.concatenate([O.hobbit_levels(a[2], t1=0.4, t_mid=0.7)[0] for a in allt]).astype(np.uint8)
            all_skip = np.concatenate([a[4] for a in allt]).astype(bool)
            cat = [all_idx, all_lvl]
            _, lv_all = O.expert_vote(all_idx, all_lvl, all_skip, E, 0.5)
            assert not np.array_equal(lv_all, cat[1])  # the vote moves some pairs
            level = lv_all[rank * T:(rank + 1) * T]
        slot = np.vectorize(lambda v: O.level_to_slot(int(v), 2))(level.astype(np.int64))
        ref = O.moe_layer(x, idx, w, slot, skip.astype(bool), recs, lays, E)
        err = O.max_rel_err(out.float().numpy(), ref)
        q.put((rank, (lo, hi), float(err), None))
        dist.destroy_process_group()
    except Exception as exc:  # report to the parent instead of hanging it
        q.put((rank, None, None, repr(exc)))


@pytest.mark.parametrize("world,vote", [(2, False), (3, False), (2, True)])
def test_ep_gloo_matches_single_process(world, vote):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, vote)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            rank, rng_, err, exc = q.get(timeout=120)
            res[rank] = (rng_, err, exc)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert sorted(res) == list(range(world))
    covered = []
    for r in range(world):
        rng_, err, exc = res[r]
        assert exc is None, exc
        assert err < 2e-3, (r, err)  # one fp16 rounding of the output
        covered.append(rng_)
    assert covered[0][0] == 0 and covered[-1][1] == E
    assert all(covered[i][1] == covered[i + 1][0] for i in range(world - 1))


def test_partition_and_owner():
    from moeb200 import ep

    for E_, G in [(64, 1), (64, 2), (64, 8), (128, 8), (512, 8), (10, 3), (7, 7)]:
        blocks = [ep.partition(E_, G, r) for r in range(G)]
        assert blocks[0][0] == 0 and blocks[-1][1] == E_
        for r in range(G - 1):
            assert blocks[r][1] == blocks[r + 1][0]
        for e in range(E_):
            r = ep.owner(e, E_, G)
            assert blocks[r][0] <= e < blocks[r][1]
    with pytest.raises(ValueError):
        ep.partition(4, 8, 0)
    with pytest.raises(ValueError):
        ep.owner(64, 64, 8)


def test_row_format_roundtrip():
    from tests import ep_util

    g = torch.Generator().manual_seed(0)
    for dt in (torch.float16, torch.bfloat16, torch.float32):
        x = torch.randn(4, 64, generator=g).to(dt)
        idx = torch.randint(0, 512, (4, 10), generator=g)
        w = torch.rand(4, 10, generator=g)
        lv = torch.randint(0, 3, (4, 10), generator=g).to(torch.uint8)
        sk = torch.randint(0, 2, (4, 10), generator=g).to(torch.uint8)
        rows = ep_util.pack_rows(x, idx, w, lv, sk)
        assert rows.shape[1] == ep_util.row_bytes(64, 10, dt) and rows.shape[1] % 16 == 0
        x2, i2, w2, l2, s2 = ep_util.unpack_rows(rows, 64, 10, dt)
        assert torch.equal(x2.view(torch.uint8), x.view(torch.uint8)) and torch.equal(i2, idx)
        assert torch.equal(w2, w) and torch.equal(l2, lv) and torch.equal(s2, sk)
