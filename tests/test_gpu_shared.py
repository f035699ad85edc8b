"""Qwen3-Next shared expert on the GPU against the oracle: sigmoid-gated SwiGLU of one record over
all tokens, added after (or instead of) the routed experts, GEMV and tcgen05 GEMM paths."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from gpu_util import TOL, act_np, make_records
from moeb200 import format as F
from moeb200 import ops
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

CASES = [  # (prec, H, I, T, act, path)
    ("int4", 2048, 512, 1, "bf16", "gemv"),
    ("int8", 2048, 512, 4, "bf16", "gemv"),
    ("bf16", 2048, 512, 8, "bf16", "gemv"),
    ("fp16", 1024, 256, 3, "fp16", "gemv"),
    ("int4", 2048, 512, 37, "fp16", "gemv"),
    ("int4", 2048, 512, 200, "bf16", "gemm"),
    ("bf16", 1024, 512, 130, "bf16", "gemm"),
    ("int8", 1024, 256, 300, "bf16", "auto"),
]
ACTS = {"bf16": torch.bfloat16, "fp16": torch.float16}


@pytest.mark.parametrize("case", CASES, ids=lambda c: "-".join(map(str, c)))
def test_shared_expert_matches_oracle(cuda_dev, case):
    prec, H, I, T, act, path = case
    dt = ACTS[act]
    lay, blobs, blobs_np = make_records(prec, H, I, 1, seed=T + H, device=cuda_dev, std=0.05)
    g = torch.Generator(device=cuda_dev).manual_seed(T)
    x = torch.randn(T, H, generator=g, device=cuda_dev).to(dt)
    wg = (torch.randn(H, generator=g, device=cuda_dev) * 0.05).to(dt)
    base = torch.randn(T, H, generator=g, device=cuda_dev).to(dt)
    ref = O.shared_expert(act_np(x), act_np(wg), blobs_np[0], lay, "bfloat16" if act == "bf16" else "float16")
    ops.set_path(path)
    try:
        out = ops.shared_expert(F.to_c(lay), blobs[0], wg, x)
        out2 = base.clone()
        ops.shared_expert(F.to_c(lay), blobs[0], wg, x, out=out2, add=True)
    finally:
        ops.set_path("auto")
    assert O.max_rel_err(act_np(out), ref) < TOL, O.max_rel_err(act_np(out), ref)
    assert O.max_rel_err(act_np(out2), act_np(base) + ref) < TOL


# -- shared expert folded into the routed launches (router_shared + an expert table of E + 1) ---------
FOLD_CASES = [  # (precs, layer precision, H, I, E, k, T, act, path)
    (["int8", "int4"], "int8", 2048, 512, 512, 10, 1, "bf16", "auto"),
    (["int8", "int4"], "int4", 2048, 512, 512, 10, 1, "bf16", "ws"),
    (["fp16", "int4"], "fp16", 2048, 512, 64, 8, 7, "fp16", "gemv"),
    (["int4"], "int4", 1024, 512, 32, 4, 300, "bf16", "auto"),
]


@pytest.mark.parametrize("case", FOLD_CASES, ids=lambda c: "-".join(map(str, c[1:])))
def test_folded_shared_expert_matches_oracle(cuda_dev, case):
    from gpu_util import emulate_router_logits
    from moeb200.runtime import B200Runtime

    precs, lp, H, I, E, k, T, act, path = case
    dt = ACTS[act]
    dts = "bfloat16" if act == "bf16" else "float16"
    lays = {p: F.record_layout(p, H, I) for p in precs}
    slot = precs.index(lp)
    P = len(precs)
    level = slot if P >= 3 else (0 if slot == 0 else 2)
    g = torch.Generator(device=cuda_dev).manual_seed(E + T)
    recs = []
    for _ in range(E + 1):  # E routed experts, then the shared MLP
        gu = torch.randn(2 * I, H, generator=g, device=cuda_dev) * 0.03
        dn = torch.randn(H, I, generator=g, device=cuda_dev) * 0.03
        recs.append(F.encode_record(lays[lp], gu, dn))
    pol = ops.PolicySpec("lo" if slot else "hi")
    rt = B200Runtime(precs, lays, E + 1, cuda_dev, pol, layers=[0])
    for e in range(E + 1):
        rt.add_record(0, e, lp, recs[e])
    x = torch.randn(T, H, generator=g, device=cuda_dev).to(dt)
    wr = (torch.randn(E, H, generator=g, device=cuda_dev) * 0.05).to(dt)
    wg = (torch.randn(H, generator=g, device=cuda_dev) * 0.05).to(dt)
    wr_ext = torch.cat([wr, wg[None]]).contiguous()
    _, w, idx, lvl, skip = ops.router(x, wr_ext, k, True, None, pol.to_c(0), want_probs=False, shared_level=level)
    # the routed columns equal the plain router's; the last column is the shared pair
    _, w0, idx0, lvl0, _ = ops.router(x, wr, k, True, None, pol.to_c(0), want_probs=False)
    assert torch.equal(idx[:, :k], idx0) and torch.equal(w[:, :k], w0) and torch.equal(lvl[:, :k], lvl0)
    assert bool((idx[:, k] == E).all()) and bool((lvl[:, k] == level).all()) and bool((skip[:, k] == 0).all())
    gl = O.round_to(emulate_router_logits(act_np(x), act_np(wg[None]), dts)[:, 0], dts)
    sig = (1.0 / (1.0 + np.exp(-gl.astype(np.float32)))).astype(np.float32)
    assert np.allclose(w[:, k].cpu().numpy(), sig, rtol=1e-6, atol=1e-7)
    ops.set_path(path)
    try:
        out = ops.experts_forward(rt._ctables[0], x, idx, w, lvl, skip, miss=rt.miss)
    finally:
        ops.set_path("auto")
    assert int(rt.miss.item()) == 0
    recs_np = [b.cpu().numpy() for b in recs]
    routed = O.moe_layer(act_np(x), idx0.cpu().numpy(), w0.cpu().numpy(), None, None, [recs_np[:E]], [lays[lp]], E)
    ref = routed + O.shared_expert(act_np(x), act_np(wg), recs_np[E], lays[lp], dts)
    assert O.max_rel_err(act_np(out), ref) < TOL, O.max_rel_err(act_np(out), ref)
