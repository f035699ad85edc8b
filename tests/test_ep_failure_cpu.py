"""Failure detection of the expert-parallel exchange on CPU gloo ranks (world size 2), made on the
host, with no GPU involved:

* a rank that raises in the middle of a layer (its expert step fails after the dispatch) and
  leaves: the surviving rank's combine collective ends with PeerFailure instead of hanging;
* a stalled rank that never enters the layer: the surviving rank's dispatch collective ends with
  PeerFailure after the process group's short timeout.

In both cases the surviving rank's ExpertParallel then refuses the next layer at once (no further
collective is entered). The reference runs on one GPU and has no exchange to fail (moelab switches
to its torch path on a kernel exception, moelab/runtime.py:346-348)."""

from __future__ import annotations

import datetime
import socket
import sys
import time
from pathlib import Path

import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
PG_TIMEOUT_S = 4.0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, mode: str, q):
    sys.path[:0] = [str(ROOT), str(ROOT / "moe-offload-lab_b200")]
    import torch
    import torch.distributed as dist

    from moeb200 import ep
    from tests import ep_util
    from tests.test_ep_cpu import E, _model, _tokens

    class FailingOps(ep_util.CpuOps):
        def local(self, *args, **kw):
            raise RuntimeError("expert step failed on this rank")

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=PG_TIMEOUT_S))
    lays, recs, wr = _model()
    lo, hi = ep.partition(E, world, rank)
    own = [[r if lo <= e < hi else None for e, r in enumerate(rs)] for rs in recs]
    rt = ep_util.CpuRuntime(E, lays, own, 2)
    faulty = rank == world - 1
    par = ep.ExpertParallel(rt, ops=FailingOps() if faulty and mode == "raise" else ep_util.CpuOps())
    x, idx, w, level, skip = _tokens(rank, wr)
    args = (torch.from_numpy(x).half(), torch.from_numpy(idx), torch.from_numpy(w), torch.from_numpy(level),
            torch.from_numpy(skip))
    if faulty and mode == "stall":
        q.put((rank, "stalling", None, None))
        time.sleep(10 * PG_TIMEOUT_S)  # never joins; the parent ends this process
        return
    t0 = time.perf_counter()
    try:
        par.run_layer(0, *args)
        q.put((rank, "completed", time.perf_counter() - t0, None))
        return
    except ep.PeerFailure as exc:
        first = ("PeerFailure", time.perf_counter() - t0, str(exc))
    except Exception as exc:  # the failing rank: report and leave without tearing the group down
        q.put((rank, type(exc).__name__, time.perf_counter() - t0, str(exc)))
        return
    t1 = time.perf_counter()
    try:
        par.run_layer(0, *args)
        second = ("completed", None)
    except ep.PeerFailure as exc:
        second = ("PeerFailure", time.perf_counter() - t1)
    q.put((rank, first[0], first[1], (first[2], second)))


def _run(mode: str, world: int = 2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            rank, kind, dt, info = q.get(timeout=180)
            res[rank] = (kind, dt, info)
    finally:
        for p in procs:
            p.join(timeout=5)
            if p.is_alive():
                p.kill()  # the stalled rank (by its own process handle)
                p.join(timeout=5)
    return res


def test_rank_that_raises_mid_layer_fails_the_peer_fast():
    res = _run("raise")
    assert res[1][0] == "RuntimeError" and "expert step failed" in res[1][2]
    kind, dt, (msg, second) = res[0]
    assert kind == "PeerFailure", res[0]
    assert "combine all_to_all" in msg  # the dispatch went through; the combine lost its peer
    assert dt < 60, dt
    assert second[0] == "PeerFailure" and second[1] < 1.0  # refused at once, no collective


def test_stalled_peer_hits_the_group_timeout():
    res = _run("stall")
    assert res[1][0] == "stalling"
    kind, dt, (msg, second) = res[0]
    assert kind == "PeerFailure", res[0]
    assert "dispatch all_gather" in msg
    assert PG_TIMEOUT_S * 0.5 <= dt < PG_TIMEOUT_S * 6, dt  # ended by the timeout, not by the peer
    assert second[0] == "PeerFailure" and second[1] < 1.0
