"""The decode step as it is measured: router -> precision mask -> dispatch -> expert kernels for
several layers, captured in ONE CUDA graph (programmatic-dependent-launch edges between the
library's kernels, counters zeroed by the kernels themselves) and replayed with new inputs copied
into the captured buffers. Every replay's routing must be bit-exact and every layer's output within
the layer tolerance of the oracle (the reference's fixed-table graph path is tested against its
eager path the same way: moelab tests/test_kernels.py:63-97, moelab/fullgraph.py:149-188).

Also: a graph captured at a small batch still replays correctly after a larger eager call grew the
library's cached workspace."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from moeb200 import ops
from moeb200.runtime import B200Runtime
from oracle import moe_oracle as O

from gpu_util import TOL, act_np, emulate_router_logits, layer_records

pytestmark = pytest.mark.gpu

H, I, E, K = 2048, 1024, 32, 8
PRECS = ["fp16", "int4"]
THR = 0.1


class Step:
    """L layers: fused router (+ threshold mask) -> experts -> residual add, on fixed buffers."""

    def __init__(self, dev, L: int, T: int, seed: int):
        self.L, self.T = L, T
        self.lays = {}
        self.recs = []
        self.rt = None
        g = torch.Generator(device=dev).manual_seed(seed)
        for li in range(L):
            lays, recs = layer_records(PRECS, H, I, E, seed=seed * 10 + li, device=dev, std=0.02)
            self.lays = lays
            self.recs.append(recs)
        self.rt = B200Runtime(PRECS, self.lays, E, dev, ops.PolicySpec("threshold", thr=THR), layers=range(L))
        for li in range(L):
            for p in PRECS:
                for e in range(E):
                    self.rt.add_record(li, e, p, self.recs[li][p][e])
        self.wr = [(torch.randn(E, H, generator=g, device=dev) * 0.02).half() for _ in range(L)]
        self.pols = [self.rt.policy.to_c(li) for li in range(L)]
        self.bufs = [dict(w=torch.empty(T, K, device=dev), idx=torch.empty(T, K, dtype=torch.int64, device=dev),
                          level=torch.empty(T, K, dtype=torch.uint8, device=dev),
                          skip=torch.empty(T, K, dtype=torch.uint8, device=dev)) for _ in range(L)]
        self.xs = [torch.zeros(T, H, dtype=torch.float16, device=dev) for _ in range(L + 1)]
        self.outs = [torch.zeros(T, H, dtype=torch.float16, device=dev) for _ in range(L)]

    def __call__(self):
        for li in range(self.L):
            b = self.bufs[li]
            ops.router(self.xs[li], self.wr[li], K, False, None, self.pols[li], want_probs=False, out=b)
            ops.experts_forward(self.rt._ctables[li], self.xs[li], b["idx"], b["w"], b["level"], b["skip"],
                                out=self.outs[li], miss=self.rt.miss)
            torch.add(self.xs[li], self.outs[li], out=self.xs[li + 1])

    def check_against_oracle(self):
        """Per layer: routing bit-exact (the kernel's documented logit order, then the oracle's
        softmax / top-k / mask), expert output within TOL of the oracle layer."""
        for li in range(self.L):
            x = act_np(self.xs[li])
            b = self.bufs[li]
            logits = emulate_router_logits(x, act_np(self.wr[li]), "float16")
            _, o_w, o_idx = O.topk_from_logits(logits, K, False)
            assert np.array_equal(b["idx"].cpu().numpy(), o_idx), li
            assert np.allclose(b["w"].cpu().numpy(), o_w, rtol=1e-5, atol=1e-8), li
            o_lvl, o_skip = O.threshold_levels(b["w"].cpu().numpy(), THR)
            assert np.array_equal(b["level"].cpu().numpy(), o_lvl), li
            assert np.array_equal(b["skip"].cpu().numpy().astype(bool), o_skip), li
            slot = np.vectorize(lambda v: O.level_to_slot(int(v), len(PRECS)))(o_lvl.astype(np.int64))
            recs_np = [[r.cpu().numpy() for r in self.recs[li][p]] for p in PRECS]
            ref = O.moe_layer(x, o_idx, b["w"].cpu().numpy(), slot, o_skip, recs_np, [self.lays[p] for p in PRECS], E)
            err = O.max_rel_err(act_np(self.outs[li]), ref)
            assert err < TOL, (li, err)


def _capture(step):
    step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    with torch.cuda.graph(g):
        step()
    torch.cuda.synchronize()
    return g


@pytest.mark.parametrize("path", ["gemv", "decode", "ws"])
@pytest.mark.parametrize("T", [1, 64])
def test_captured_step_replays_match_oracle(cuda_dev, path, T):
    ops.set_path(path)
    try:
        step = Step(cuda_dev, L=2, T=T, seed=3 + T)
        g = _capture(step)
        gen = torch.Generator(device=cuda_dev).manual_seed(100 + T)
        for rep in range(3):
            step.xs[0].copy_(torch.randn(T, H, generator=gen, device=cuda_dev).half())
            g.replay()
            torch.cuda.synchronize()
            step.check_against_oracle()
        assert int(step.rt.miss.item()) == 0
        del g
    finally:
        ops.set_path("auto")


@pytest.mark.parametrize("path", ["gemv", "decode", "ws"])
def test_graph_survives_workspace_growth(cuda_dev, path):
    # capture at T=8, grow the cached workspaces with an eager T=64 layer, replay the T=8 graph
    ops.set_path(path)
    # start from empty caches so the T=8 capture gets buffers that the T=64 call must outgrow (the
    # buffers cached so far are retired, not freed: graphs of earlier tests keep them)
    ops._RETIRED.extend(ops._WS.values())
    ops._WS.clear()
    try:
        small = Step(cuda_dev, L=1, T=8, seed=21)
        g = _capture(small)
        big = Step(cuda_dev, L=1, T=64, seed=22)
        big.xs[0].copy_(torch.randn(64, H, device=cuda_dev).half())
        big()
        torch.cuda.synchronize()
        big.check_against_oracle()
        small.xs[0].copy_(torch.randn(8, H, device=cuda_dev).half())
        g.replay()
        torch.cuda.synchronize()
        small.check_against_oracle()
        del g
    finally:
        ops.set_path("auto")
