"""Expert-parallel kernels on the GPU: exchange rows byte-exact against the torch mirror of the
format, owned-expert partial sums + rank-order combine equal to the single-GPU layer and the
oracle, and (with two or more GPUs) the expert-parallel layer on 2 ranks with the NCCL and with the
peer-memory exchange."""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from gpu_util import TOL, act_np, layer_records
from moeb200 import B200Runtime, ops
from oracle import moe_oracle as O
from tests import ep_util

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("k", [8, 10])
def test_ep_pack_unpack_bytes(cuda_dev, dt, k):
    g = torch.Generator(device=cuda_dev).manual_seed(k)
    T, H = 37, 256
    x = torch.randn(T, H, generator=g, device=cuda_dev).to(dt)
    idx = torch.randint(0, 512, (T, k), generator=g, device=cuda_dev)
    w = torch.rand(T, k, generator=g, device=cuda_dev)
    lv = torch.randint(0, 3, (T, k), generator=g, device=cuda_dev).to(torch.uint8)
    sk = torch.randint(0, 2, (T, k), generator=g, device=cuda_dev).to(torch.uint8)
    rows = torch.full((T, ops.ep_row_bytes(H, k, dt)), 0xAB, dtype=torch.uint8, device=cuda_dev)
    ops.ep_pack(x, idx, w, lv, sk, rows)
    assert torch.equal(rows.cpu(), ep_util.pack_rows(x.cpu(), idx.cpu(), w.cpu(), lv.cpu(), sk.cpu()))
    x2, i2, w2 = torch.empty_like(x), torch.empty_like(idx), torch.empty_like(w)
    l2, s2 = torch.empty_like(lv), torch.empty_like(sk)
    ops.ep_unpack(rows, H, k, dt, x2, i2, w2, l2, s2)
    assert torch.equal(x2.view(torch.uint8), x.view(torch.uint8)) and torch.equal(i2, idx)
    assert torch.equal(w2, w) and torch.equal(l2, lv) and torch.equal(s2, sk)
    # level/skip NULL on pack write zeros
    ops.ep_pack(x, idx, w, None, None, rows)
    _, _, _, l3, s3 = ep_util.unpack_rows(rows.cpu(), H, k, dt)
    assert int(l3.sum()) == 0 and int(s3.sum()) == 0


@pytest.mark.parametrize("G", [2, 4])
@pytest.mark.parametrize("path", ["gemv", "gemm"])
def test_partial_sums_combine_to_layer(cuda_dev, G, path):
    H, I, E, k, T = 256, 128, 16, 4, 48
    precs = ["fp16", "int4"]
    lays, recs = layer_records(precs, H, I, E, seed=21, device=cuda_dev, std=0.05)
    rt = B200Runtime(precs, lays, E, cuda_dev, ops.PolicySpec("threshold", thr=0.3), layers=[0])
    for p in precs:
        for e in range(E):
            rt.add_record(0, e, p, recs[p][e])
    g = torch.Generator(device=cuda_dev).manual_seed(3)
    x = torch.randn(T, H, generator=g, device=cuda_dev).half()
    wv, idx = torch.topk(torch.randn(T, E, generator=g, device=cuda_dev).softmax(-1), k, dim=-1)
    lvl, skip = rt.levels(0, wv)
    ops.set_path(path)
    try:
        full = rt.run_layer(0, x, idx, wv, level=lvl, skip=skip)
        parts = torch.empty(G, T, H, dtype=torch.float32, device=cuda_dev)
        table = rt._ctables[0]
        for r in range(G):
            lo, hi = r * E // G, (r + 1) * E // G
            ops.experts_forward_part(table, lo, hi, x, idx, wv, lvl, skip, part=parts[r], miss=rt.miss)
        out = torch.empty_like(x)
        ops.combine_parts(parts, out)
    finally:
        ops.set_path("auto")
    assert int(rt.miss.item()) == 0
    slot = np.vectorize(lambda v: O.level_to_slot(int(v), 2))(lvl.cpu().numpy().astype(np.int64))
    recs_np = [[b.cpu().numpy() for b in recs[p]] for p in precs]
    ref = O.moe_layer(act_np(x), idx.cpu().numpy(), wv.cpu().numpy(), slot, skip.cpu().numpy().astype(bool), recs_np,
                      [lays[p] for p in precs], E)
    assert O.max_rel_err(act_np(out), ref) < TOL
    # the partial sums only reorder fp32 additions: the layer agrees to an output rounding or two
    assert O.max_rel_err(act_np(out), act_np(full)) < 4e-3
    # each part holds only its own experts' pairs: part r == oracle restricted to its block
    for r in range(G):
        lo, hi = r * E // G, (r + 1) * E // G
        idn = idx.cpu().numpy()
        sk = skip.cpu().numpy().astype(bool) | (idn < lo) | (idn >= hi)
        ref_r = O.moe_layer(act_np(x), idn, wv.cpu().numpy(), slot, sk, recs_np, [lays[p] for p in precs], E)
        assert O.max_rel_err(parts[r].cpu().numpy(), ref_r) < TOL


def test_combine_parts_order_and_add(cuda_dev):
    g = torch.Generator(device=cuda_dev).manual_seed(0)
    parts = torch.randn(3, 5, 64, generator=g, device=cuda_dev)
    base = torch.randn(5, 64, generator=g, device=cuda_dev).to(torch.bfloat16)
    out = base.clone()
    ops.combine_parts(parts, out, add=True)
    ref = ((parts[0] + parts[1]) + parts[2])
    ref = (base.float() + ref).to(torch.bfloat16)
    assert torch.equal(out, ref)
    o32 = torch.empty(5, 64, device=cuda_dev)
    ops.combine_parts(parts, o32)
    assert torch.equal(o32, (parts[0] + parts[1]) + parts[2])


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("exchange", ["nccl", "p2p", "nccl_cold"])
def test_expert_parallel_two_ranks(tmp_path, exchange):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=f"{ROOT}:{ROOT / 'moe-offload-lab_b200'}")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           str(ROOT / "tests" / "ep_worker.py"), str(tmp_path), exchange]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    for rank in range(2):
        res = json.loads((tmp_path / f"rank{rank}.json").read_text())
        assert res["exchange"] == exchange
        assert res["err_oracle"] < TOL, res
        assert res["err_single"] < 4e-3, res
        assert res["err_repeat"] < 4e-3, res  # the second call reuses the exchange buffers
        assert res["miss"] == 0 and res["status"] == 0, res
        if exchange == "nccl_cold":
            assert res["uploads"] > 0, res
