"""Qwen3-Next shared expert on the GPU against the oracle: sigmoid-gated SwiGLU of one record over
all tokens, added after (or instead of) the routed experts, GEMV and tcgen05 GEMM paths."""

from __future__ import annotations

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
