"""One rank of the 2-GPU expert-parallel test (launched by tests/test_gpu_ep.py through
torch.distributed.run): every rank holds only its experts' records, runs the EP layer on its own
tokens, and compares with the single-GPU layer over all experts and with the oracle. Mode
"nccl_cold": the NCCL exchange with a third of each rank's experts held on the host (ColdExperts),
uploaded from the gathered routing of both ranks."""

from __future__ import annotations

import datetime
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parents[1]
sys.path[:0] = [str(ROOT), str(ROOT / "moe-offload-lab_b200"), str(ROOT / "tests")]

from gpu_util import act_np, layer_records  # noqa: E402
from moeb200 import B200Runtime, ops  # noqa: E402
from moeb200.ep import ExpertParallel  # noqa: E402
from oracle import moe_oracle as O  # noqa: E402


def main():
    out_dir = Path(sys.argv[1])
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    H, I, E, k, T = 256, 128, 16, 4, 24
    precs = ["fp16", "int4"]
    lays, recs = layer_records(precs, H, I, E, seed=31, device=dev, std=0.05)  # same on every rank
    pol = ops.PolicySpec("threshold", thr=0.3)
    full_rt = B200Runtime(precs, lays, E, dev, pol, layers=[0])
    ep_rt = B200Runtime(precs, lays, E, dev, pol, layers=[0])
    mode = sys.argv[2] if len(sys.argv) > 2 else "p2p"
    ep = ExpertParallel(ep_rt, exchange="nccl" if mode == "nccl_cold" else mode)
    for p in precs:
        for e in range(E):
            full_rt.add_record(0, e, p, recs[p][e])
            if ep.owns(e):
                ep_rt.add_record(0, e, p, recs[p][e])
    if mode == "nccl_cold":
        from moeb200.cold import ColdExperts

        owned_cold = [e for e in range(ep.e_lo, ep.e_hi) if e % 3 == 1]
        cold = ColdExperts(ep_rt, {p: len(owned_cold) for p in precs})
        for e in owned_cold:
            for p in precs:
                cold.add_cold(0, e, p, recs[p][e].cpu())
        ep.cold = cold
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    x = torch.randn(T, H, generator=g, device=dev).half()
    wv, idx = torch.topk(torch.randn(T, E, generator=g, device=dev).softmax(-1), k, dim=-1)
    lvl, skip = full_rt.levels(0, wv)
    out = ep.run_layer(0, x, idx, wv, lvl, skip)
    out2 = ep.run_layer(0, x, idx, wv, lvl, skip).clone()  # a second call reuses the exchange buffers
    single = full_rt.run_layer(0, x, idx, wv, level=lvl, skip=skip)
    torch.cuda.synchronize()
    slot = np.vectorize(lambda v: O.level_to_slot(int(v), 2))(lvl.cpu().numpy().astype(np.int64))
    recs_np = [[b.cpu().numpy() for b in recs[p]] for p in precs]
    ref = O.moe_layer(act_np(x), idx.cpu().numpy(), wv.cpu().numpy(), slot, skip.cpu().numpy().astype(bool), recs_np,
                      [lays[p] for p in precs], E)
    res = {"rank": rank, "owned": [ep.e_lo, ep.e_hi], "exchange": mode,
           "uploads": ep.cold.uploads if ep.cold is not None else 0,
           "err_oracle": O.max_rel_err(act_np(out), ref), "err_single": O.max_rel_err(act_np(out), act_np(single)),
           "err_repeat": O.max_rel_err(act_np(out2), act_np(out)), "miss": int(ep_rt.miss.item()),
           "status": ep.status() if ep.exchange == "p2p" else 0}
    (out_dir / f"rank{rank}.json").write_text(json.dumps(res))
    dist.barrier()
    ep.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
