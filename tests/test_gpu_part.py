"""Partial expert sums (moeb200_experts_forward_part, the expert-parallel building block) for calls of
up to 8 tokens, which take the warp-streamed GEMV: the experts split into G contiguous blocks, each
block's fp32 partial computed on its own, combined in block order, against the whole layer in one
call and against the oracle (needs a B200)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from moeb200 import _lib, ops
from moeb200.runtime import B200Runtime
from oracle import moe_oracle as O

from gpu_util import act_np, layer_records

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("G", [2, 3])
@pytest.mark.parametrize("T", [1, 6])
def test_partials_of_small_calls_add_up_to_the_layer(cuda_dev, T, G):
    H, I, E, k = 512, 512, 24, 4
    precs = ["fp16", "int4"]
    lays, recs = layer_records(precs, H, I, E, seed=17, device=cuda_dev, std=0.05)
    rt = B200Runtime(precs, lays, E, cuda_dev, ops.PolicySpec("threshold", thr=0.3), layers=[0])
    for p in precs:
        for e in range(E):
            rt.add_record(0, e, p, recs[p][e])
    g = torch.Generator(device=cuda_dev).manual_seed(23)
    x = torch.randn(T, H, generator=g, device=cuda_dev).half()
    wv, idx = torch.topk(torch.randn(T, E, generator=g, device=cuda_dev).softmax(-1), k, dim=-1)
    lvl, skip = rt.levels(0, wv)
    table = rt._ctables[0]
    whole = ops.experts_forward(table, x, idx, wv, lvl, skip)
    bounds = [E * r // G for r in range(G + 1)]
    parts = torch.empty(G, T, H, dtype=torch.float32, device=cuda_dev)
    for r in range(G):
        ops.experts_forward_part(table, bounds[r], bounds[r + 1], x, idx, wv, lvl, skip, part=parts[r])
        assert _lib.lib().moeb200_path_used() == 4  # the warp-streamed GEMV
    out = torch.empty_like(x)
    ops.combine_parts(parts, out)
    torch.cuda.synchronize()
    # the blocks' sums differ from the whole layer's only in the fp32 summation order
    assert O.max_rel_err(act_np(out), act_np(whole)) < 1e-3
    slot = np.vectorize(lambda v: O.level_to_slot(int(v), 2))(lvl.cpu().numpy().astype(np.int64))
    ref = O.moe_layer(act_np(x), idx.cpu().numpy(), wv.cpu().numpy(), slot, skip.cpu().numpy().astype(bool),
                      [[b.cpu().numpy() for b in recs[p]] for p in precs], [lays[p] for p in precs], E)
    assert O.max_rel_err(act_np(out), ref) < 1e-2
